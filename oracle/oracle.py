"""CPU oracle for the FP8 decode/prefill custom-op path — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this module, and only as the checker (or, for the CPU baseline, as the
thing timed on the host cores).  The product path (esimd_learning_b200 and
libcek_b200.so) never calls it; there is no CPU fallback.

It restates, in torch fp32 on the CPU, the math the reference's own tests use
as their oracle, and the kernel semantics where the tests are silent:

* GEMV / GEMM: `input.float() @ weight_fp8.to(fp16).float().T * scale`
  (tests/test_gemv_fp8.py:31-32, :58-59, :349-350; tests/test_gemm_fp8.py:35-36),
  with the scale applied after the fp32 reduction as the kernel does
  (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:77).
* add + RMSNorm: tests/test_fused_add_rms_norm_batched_fp8.py:7-27, with the
  kernel's rounding points: the residual is stored in the I/O type, the sum of
  squares runs over the unrounded sum, the normalised value is computed from
  the rounded residual (csrc/xpu/esimd_kernels/fused_add_rms_norm_batched.h:
  32-50, 56-62).
* GeLU(tanh)-and-mul, q/k-norm + RoPE, per-token quantisation and the
  per-token x per-channel FP8 GEMM have no reference implementation; they are
  restated from their published definitions (tanh-GeLU, RMSNorm, rotary
  embedding with vLLM's cos/sin cache layout, e4m3 round-to-nearest-even).
  Parity for these rows is pinned to these definitions only.

FP8 decoding uses exact tables built from the format definitions (OCP FP8:
e4m3fn and e5m2), pinned in tests against torch's own float8 conversion for
all 256 codes and against the reference kernel's bit-trick decode
(fp8_GEMV_v2.h:15-38) on every normal code.
"""
from __future__ import annotations

import math

import torch

E4M3, E5M2 = 0, 1
E4M3_MAX = 448.0


# ---- FP8 decoding --------------------------------------------------------------

def fp8_decode_table(fmt: int) -> torch.Tensor:
    """float32[256]: exact value of every FP8 code (NaN codes -> NaN)."""
    vals = []
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        if fmt == E4M3:
            e, m = (b >> 3) & 0xF, b & 0x7
            if e == 0xF and m == 0x7:
                v = math.nan
            elif e == 0:
                v = s * (m / 8.0) * 2.0 ** -6
            else:
                v = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
        else:
            e, m = (b >> 2) & 0x1F, b & 0x3
            if e == 0x1F:
                v = s * math.inf if m == 0 else math.nan
            elif e == 0:
                v = s * (m / 4.0) * 2.0 ** -14
            else:
                v = s * (1.0 + m / 4.0) * 2.0 ** (e - 15)
        vals.append(v)
    return torch.tensor(vals, dtype=torch.float32)


def fp8_decode_table_reference_kernel(fmt: int) -> torch.Tensor:
    """float32[256]: the reference kernel's decode (fp8_GEMV_v2.h:15-38):
    e4m3 -> fp16 bits sign<<15 | (exp+8)<<10 | mant<<7, e5m2 -> sign<<15 |
    exp<<10 | mant<<8, exponent-0 codes flushed to signed zero."""
    out = torch.empty(256, dtype=torch.int32)
    for b in range(256):
        s = (b >> 7) & 1
        if fmt == E4M3:
            e, m = (b >> 3) & 0xF, b & 0x7
            bits = (s << 15) | ((e + 8) << 10) | (m << 7)
        else:
            e, m = (b >> 2) & 0x1F, b & 0x3
            bits = (s << 15) | (e << 10) | (m << 8)
        if e == 0:
            bits = s << 15
        out[b] = bits
    return out.to(torch.int16).view(torch.float16).float()


_TABLES: dict[int, torch.Tensor] = {}


def fp8_decode(codes: torch.Tensor, fmt: int) -> torch.Tensor:
    """Decode FP8 codes (any 8-bit dtype, CPU) to float32 exactly."""
    if fmt not in _TABLES:
        _TABLES[fmt] = fp8_decode_table(fmt)
    return _TABLES[fmt][codes.contiguous().view(torch.uint8).long()]


def fp8_format_of(w: torch.Tensor) -> int:
    return E5M2 if w.dtype == torch.float8_e5m2 else E4M3


# ---- GEMV / GEMM ----------------------------------------------------------------

def gemv_fp8(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, out_dtype=None,
             fmt: int | None = None) -> torch.Tensor:
    """y[M, N] = out_dtype( (x.f32 @ deq(w).T) * scale ), scale fp16/fp32 [N] or scalar.

    Restates tests/test_gemv_fp8.py:58-59 (per-N) and :349-350 (per-tensor).
    """
    fmt = fp8_format_of(w) if fmt is None else fmt
    out_dtype = out_dtype or x.dtype
    K = w.shape[-1]
    wf = fp8_decode(w.cpu(), fmt).reshape(-1, K)
    xf = x.cpu().float().reshape(-1, K)
    s = scale.cpu().float().reshape(-1)
    y = (xf @ wf.T) * (s if s.numel() > 1 else s[0])
    return y.to(out_dtype)


def gemm_fp8_scaled(aq: torch.Tensor, a_scale: torch.Tensor, bq: torch.Tensor,
                    b_scale: torch.Tensor, out_dtype=torch.float16) -> torch.Tensor:
    """Y = out_dtype( (deq(aq) @ deq(bq).T) * a_scale[:, None] * b_scale[None, :] )."""
    af = fp8_decode(aq.cpu(), E4M3).reshape(aq.shape)
    bf = fp8_decode(bq.cpu(), E4M3).reshape(bq.shape)
    y = (af @ bf.T) * a_scale.cpu().float().reshape(-1, 1) * b_scale.cpu().float().reshape(1, -1)
    return y.to(out_dtype)


def quant_fp8_per_token(a: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """s[m] = max(amax|a[m]|, 1e-12) / 448;  aq = e4m3_rne(clamp(a / s, -448, 448))."""
    af = a.cpu().float()
    s = af.abs().amax(dim=-1).clamp(min=1e-12) / E4M3_MAX
    q = (af / s.unsqueeze(-1)).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q, s


# ---- residual add + RMSNorm --------------------------------------------------------

def add_rmsnorm(hidden: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (new_residual, normed), both in the I/O dtype (kernel rounding points)."""
    dt = hidden.dtype
    s = hidden.cpu().float() + residual.cpu().float()
    r = s.to(dt)
    inv = torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    normed = (r.float() * inv * weight.cpu().float()).to(dt)
    return r, normed


def add_rmsnorm_gemv_fp8(hidden, residual, gamma, eps, w, scale):
    """(new_residual, y): add+RMSNorm, round the normalised row to the I/O
    dtype, then the FP8 GEMV, i.e. the two reference ops composed."""
    r, normed = add_rmsnorm(hidden, residual, gamma, eps)
    return r, gemv_fp8(normed, w, scale, out_dtype=hidden.dtype)


# ---- GeLU-and-mul, q/k-norm + RoPE ------------------------------------------------------

def gelu_and_mul(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1] // 2
    xf = x.cpu().float()
    g, u = xf[..., :d], xf[..., d:]
    act = 0.5 * g * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (g + 0.044715 * g.pow(3))))
    return (act * u).to(x.dtype)


def rope_cos_sin_cache(max_position: int, head_dim: int, theta: float) -> torch.Tensor:
    """fp32 [max_position, head_dim]: cos | sin halves (vLLM RotaryEmbedding layout)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1)


def qkv_norm_rope(qkv, positions, q_weight, k_weight, cos_sin_cache, num_q_heads,
                  num_kv_heads, head_dim, eps, is_neox=True) -> torch.Tensor:
    dt = qkv.dtype
    M = qkv.numel() // ((num_q_heads + 2 * num_kv_heads) * head_dim)
    x = qkv.cpu().reshape(M, num_q_heads + 2 * num_kv_heads, head_dim).clone()
    out = x.clone()
    nh = num_q_heads + num_kv_heads
    heads = x[:, :nh].float()
    w = torch.cat([q_weight.cpu().float().expand(num_q_heads, head_dim),
                   k_weight.cpu().float().expand(num_kv_heads, head_dim)])
    inv = torch.rsqrt(heads.pow(2).mean(-1, keepdim=True) + eps)
    xn = (heads * inv * w).to(dt).float()
    pos = positions.cpu().long().clamp(0, cos_sin_cache.shape[0] - 1)
    cs = cos_sin_cache.cpu()[pos]  # [M, D]
    half = head_dim // 2
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    if is_neox:
        x1, x2 = xn[..., :half], xn[..., half:]
        o = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)
    else:
        x1, x2 = xn[..., 0::2], xn[..., 1::2]
        o = torch.stack([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).flatten(-2)
    out[:, :nh] = o.to(dt)
    return out.reshape(qkv.shape)


# ---- parity metrics (north_star tolerance) -----------------------------------------------

MAX_ABS_FRAC = 1e-2   # max |out - ref| <= 1e-2 * ||ref||_inf
MEAN_REL = 2e-3       # mean |out - ref| / mean |ref| <= 2e-3


def parity(out: torch.Tensor, ref: torch.Tensor) -> dict:
    o = out.detach().cpu().float()
    r = ref.detach().cpu().float()
    err = (o - r).abs()
    ref_inf = r.abs().max().item() if r.numel() else 0.0
    mean_ref = r.abs().mean().item() if r.numel() else 0.0
    return {
        "max_abs": err.max().item() if r.numel() else 0.0,
        "ref_inf": ref_inf,
        "max_abs_frac": (err.max().item() / ref_inf) if ref_inf > 0 else 0.0,
        "mean_rel": (err.mean().item() / mean_ref) if mean_ref > 0 else 0.0,
        "finite": bool(torch.isfinite(o).all().item()),
    }


def assert_parity(out: torch.Tensor, ref: torch.Tensor, what: str = "") -> dict:
    m = parity(out, ref)
    assert m["finite"], f"{what}: non-finite output"
    assert m["max_abs_frac"] <= MAX_ABS_FRAC, f"{what}: max-abs {m}"
    assert m["mean_rel"] <= MEAN_REL, f"{what}: mean-rel {m}"
    return m


# ---- tensor-parallel decode step, unsharded -------------------------

def decode_chain(full: dict, shape, hidden, residual, attn_out, positions):
    """One decode step of the 70B-shaped layer on the unsharded weights:
    add+RMSNorm -> QKV GEMV -> q/k-norm + RoPE; add+RMSNorm -> gate_up GEMV ->
    GeLU-and-mul -> down GEMV.  Returns (out, qkv, new_residual); the sharded
    GPU step must match it (out after the all-reduce, qkv per rank shard)."""
    r1, qkv = add_rmsnorm_gemv_fp8(hidden, residual, full["gamma_attn"], shape.eps, *full["qkv"])
    cs = rope_cos_sin_cache(shape.max_position, shape.head_dim, shape.rope_theta)
    qkv = qkv_norm_rope(qkv, positions, full["q_norm"], full["k_norm"], cs, shape.num_q_heads,
                        shape.num_kv_heads, shape.head_dim, shape.eps, True)
    r2, gu = add_rmsnorm_gemv_fp8(attn_out, r1, full["gamma_mlp"], shape.eps, *full["gate_up"])
    act = gelu_and_mul(gu)
    out = gemv_fp8(act, *full["down"])
    return out, qkv, r2
