"""GeLU(tanh)-and-mul, q/k-norm + RoPE and per-token e4m3 quantisation on the
GPU against the oracle (BASELINE config 4 shapes)."""
import pytest
import torch

from esimd_learning_b200 import cabi
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,d", [(1, 28672), (16, 3584), (7, 8), (3, 1000), (2, 9), (4, 1500)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_gelu_and_mul(ext, cuda_device, M, d, io):
    torch.manual_seed(0)
    x = (torch.randn(M, 2 * d) * 2).to(io)
    out = torch.zeros(M, d, dtype=io, device=cuda_device)
    ext.esimd_gelu_and_mul(x.to(cuda_device), out)
    O.assert_parity(out, O.gelu_and_mul(x), f"M={M} d={d}")


@pytest.mark.parametrize("hq,hkv,D", [(64, 8, 128), (8, 1, 128), (16, 4, 64), (4, 2, 256)])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_qkv_norm_rope(ext, cuda_device, hq, hkv, D, neox, io):
    torch.manual_seed(1)
    M = 5
    qkv = torch.randn(M, (hq + 2 * hkv) * D).to(io)
    pos = torch.randint(0, 8192, (M,), dtype=torch.int64)
    qw = (1 + 0.1 * torch.randn(D)).to(io)
    kw = (1 + 0.1 * torch.randn(D)).to(io)
    cs = O.rope_cos_sin_cache(8192, D, 500000.0)
    ref = O.qkv_norm_rope(qkv, pos, qw, kw, cs, hq, hkv, D, 1e-6, neox)
    qd = qkv.to(cuda_device)
    ext.esimd_qkv_norm_rope(qd, pos.to(cuda_device), qw.to(cuda_device), kw.to(cuda_device),
                            cs.to(cuda_device), hq, hkv, D, 1e-6, neox)
    qc = qd.cpu()
    v0 = (hq + hkv) * D
    assert torch.equal(qc[:, v0:], qkv[:, v0:])
    O.assert_parity(qc[:, :v0], ref[:, :v0], f"hq={hq} hkv={hkv} D={D} neox={neox}")


@pytest.mark.parametrize("M,K", [(1, 4096), (2048, 4096), (13, 4096), (5, 8), (33, 1000), (7, 8192), (3, 16384), (9, 2048)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_quant_fp8_per_token_bit_exact(ext, cuda_device, M, K, io):
    torch.manual_seed(2)
    a = torch.randn(M, K).to(io)
    a[0, :] = 0 if M > 3 else a[0, :]
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.empty(M, dtype=torch.float32, device=cuda_device)
    ext.esimd_quant_fp8_per_token(a.to(cuda_device), q, s)
    rq, rs = O.quant_fp8_per_token(a)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


def test_quant_through_cabi(cuda_device):
    a = torch.randn(4, 512, dtype=torch.float16, device=cuda_device)
    q = torch.empty(4, 512, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.empty(4, dtype=torch.float32, device=cuda_device)
    cabi.call("cek_quant_fp8_per_token", cabi.ptr(a), cabi.ptr(q), cabi.ptr(s), 4, 512, cabi.CEK_F16,
              cabi.current_stream())
    torch.cuda.synchronize()
    rq, rs = O.quant_fp8_per_token(a.cpu())
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


# ---- GeLU-and-mul fused into the gate_up GEMV epilogue --------------------------

def _gated_case(M, N, K, io, seed):
    from esimd_learning_b200.workloads import make_fp8_weight
    gen = torch.Generator().manual_seed(seed)
    x = (torch.randn(M, K, generator=gen)).to(io)
    wq, sc = make_fp8_weight(2 * N, K, gen)  # gate rows [0, N), up rows [N, 2N)
    return x, wq, sc


@pytest.mark.parametrize("M,N,K", [(1, 512, 1024), (3, 1000, 4096), (8, 256, 2048), (1, 3584, 8192),
                                   (2, 1500, 14336), (8, 4096, 8192), (5, 9, 64), (12, 256, 1024),
                                   (16, 1000, 4096), (20, 256, 1024)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_gemv_gelu_mul(ext, cuda_device, M, N, K, io):
    """The gated GEMV equals the plain GEMV into [M, 2N] followed by
    esimd_gelu_and_mul, bit for bit (same GEMV sums, same rounding of gate
    and up, same pinned GeLU arithmetic), for the fused kernel (M <= 16,
    ragged N, K cut into pieces, x in tensor memory at M = 8, K = 8192, two
    token groups at M = 12, 16) and for the op's two-launch fallback
    (M = 20).  Both agree with the oracle."""
    import esimd_learning_b200 as ops

    x, wq, sc = _gated_case(M, N, K, io, seed=M * 1000 + N)
    xd, wd, sd = x.to(cuda_device), wq.to(cuda_device), sc.to(cuda_device)
    y = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    ops.esimd_gemv_fp8_gelu_mul(xd, wd, sd, y)
    gu = torch.empty(M, 2 * N, dtype=io, device=cuda_device)
    ops.esimd_gemv_fp8_pern(xd, wd, sd, gu, 2 * N, K)
    y2 = torch.empty(M, N, dtype=io, device=cuda_device)
    ops.esimd_gelu_and_mul(gu, y2)
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    O.assert_parity(y, O.gelu_and_mul(O.gemv_fp8(x, wq, sc)), f"M={M} N={N} K={K}")


@pytest.mark.parametrize("M", [1, 4, 8, 16])
def test_fused_norm_gelu_mul(ext, cuda_device, M):
    """add + RMSNorm + gated gate_up GEMV + GeLU-and-mul equals the fused-norm
    op into [M, 2N] followed by esimd_gelu_and_mul, bit for bit, including the
    residual update (M = 16: two token groups)."""
    import esimd_learning_b200 as ops
    from esimd_learning_b200.workloads import make_fp8_weight

    N, K = 1536, 4096
    gen = torch.Generator().manual_seed(M)
    h = torch.randn(M, K, generator=gen).half()
    r = torch.randn(M, K, generator=gen).half()
    gamma = (1 + 0.1 * torch.randn(K, generator=gen)).half()
    wq, sc = make_fp8_weight(2 * N, K, gen)
    dev = cuda_device
    wd, sd, gd = wq.to(dev), sc.to(dev), gamma.to(dev)
    h1, r1 = h.to(dev), r.to(dev)
    y = torch.empty(M, N, dtype=torch.float16, device=dev)
    ops.esimd_fused_add_rms_norm_gelu_mul_fp8(h1, r1, gd, 1e-6, wd, sd, y)
    h2, r2 = h.to(dev), r.to(dev)
    gu = torch.empty(M, 2 * N, dtype=torch.float16, device=dev)
    ops.esimd_fused_add_rms_norm_batched_fp8(h2, r2, gd, 1e-6, wd, sd, gu)
    y2 = torch.empty(M, N, dtype=torch.float16, device=dev)
    ops.esimd_gelu_and_mul(gu, y2)
    torch.cuda.synchronize()
    assert torch.equal(r1, r2)
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    ref_r, ref_n = O.add_rmsnorm(h, r, gamma, 1e-6)
    O.assert_parity(y, O.gelu_and_mul(O.gemv_fp8(ref_n, wq, sc)), f"M={M}")


def test_gelu_mul_output_flag_cabi(cuda_device):
    """C ABI: CEK_GEMV_GELU_MUL_OUTPUT (N = output columns, w has 2N rows)
    runs where the gated kernel fits and returns CEK_ERR_UNSUPPORTED,
    launching nothing, where it does not (M > 16, K % 64 != 0)."""
    x, wq, sc = _gated_case(2, 300, 4096, torch.float16, seed=5)
    xd, wd, sd = x.to(cuda_device), wq.to(cuda_device), sc.to(cuda_device)
    y = torch.zeros(2, 300, dtype=torch.float16, device=cuda_device)
    cabi.call("cek_gemv_fp8", cabi.ptr(xd), cabi.ptr(wd), cabi.ptr(sd), cabi.ptr(y), 2, 300, 4096, cabi.CEK_F16,
              cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, cabi.CEK_GEMV_GELU_MUL_OUTPUT,
              cabi.current_stream())
    torch.cuda.synchronize()
    O.assert_parity(y, O.gelu_and_mul(O.gemv_fp8(x, wq, sc)), "flag")
    L = cabi.lib()
    for M, K in ((17, 4096), (2, 4080)):
        xb = torch.zeros(M, K, dtype=torch.float16, device=cuda_device)
        yb = torch.zeros(M, 300, dtype=torch.float16, device=cuda_device)
        rc = L.cek_gemv_fp8(cabi.ptr(xb), cabi.ptr(wd), cabi.ptr(sd), cabi.ptr(yb), M, 300, K, cabi.CEK_F16,
                            cabi.CEK_F16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, cabi.CEK_GEMV_GELU_MUL_OUTPUT,
                            cabi.current_stream())
        assert rc == cabi.CEK_ERR_UNSUPPORTED


@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_quant_every_16bit_value_many_scales(ext, cuda_device, io):
    """Every finite positive and negative 16-bit value, in rows whose amax
    (and so scale) differ, against torch's IEEE division: the codes and the
    scales must agree bit for bit."""
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16)
    vals = bits.view(io).float()
    vals = vals[torch.isfinite(vals)]
    K = 4096
    vals = vals[: (vals.numel() // K) * K].reshape(-1, K)
    g = torch.Generator().manual_seed(7)
    rows = []
    for i in range(vals.shape[0]):
        r = vals[i].clone()
        # a per-row amax drawn across 12 octaves, so the scales differ widely
        amax = float(2.0 ** torch.randint(-6, 6, (1,), generator=g).item()) * (1 + torch.rand(1, generator=g).item())
        r = torch.where(r.abs() > amax, torch.zeros_like(r), r)
        r[0] = amax
        rows.append(r)
    a = torch.stack(rows).to(io)
    M = a.shape[0]
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=cuda_device)
    s = torch.empty(M, dtype=torch.float32, device=cuda_device)
    ext.esimd_quant_fp8_per_token(a.to(cuda_device), q, s)
    rq, rs = O.quant_fp8_per_token(a)
    assert torch.equal(s.cpu(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_quant_near_e4m3_ties_many_scales(ext, cuda_device, io):
    """Values placed on and next to the e4m3 rounding midpoints of a / s,
    over 4096 rows whose scales span the 16-bit type's whole range (plus a
    row with an infinite input and one with a NaN): the kernel's quotient must round to the
    same code as torch's IEEE division, bit for bit, and the scales agree."""
    g = torch.Generator().manual_seed(11)
    M, K = 4096, 1024
    lo, hi = (-20, 15) if io == torch.float16 else (-120, 120)
    amax = 2.0 ** torch.randint(lo, hi, (M, 1), generator=g).double() * (1 + torch.rand(M, 1, generator=g, dtype=torch.float64))
    s = (amax.float() / 448.0).double()
    # e4m3 codes 0..447 and the midpoints between neighbouring codes
    codes = torch.arange(0, 256, dtype=torch.uint8).view(torch.float8_e4m3fn).double()
    codes = codes[torch.isfinite(codes) & (codes >= 0)].sort().values
    mids = (codes[1:] + codes[:-1]) / 2
    pick = torch.randint(0, mids.numel(), (M, K), generator=g)
    sign = torch.where(torch.rand(M, K, generator=g) < 0.5, -1.0, 1.0).double()
    a = (mids[pick] * sign * s).to(io)
    # nudge a third of them one 16-bit step either way
    bits = a.view(torch.int16)
    nudge = torch.randint(-1, 2, (M, K), generator=g).to(torch.int16)
    a = (bits + nudge).view(io)
    a[:, 0] = amax.squeeze(1).to(io)
    a = torch.where(torch.isfinite(a.float()), a, torch.zeros_like(a))
    a[M - 1, 5] = float("inf")
    a[M - 2, 9] = float("nan")  # torch's amax propagates NaN: scale and codes NaN
    q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=cuda_device)
    sc = torch.empty(M, dtype=torch.float32, device=cuda_device)
    ext.esimd_quant_fp8_per_token(a.to(cuda_device), q, sc)
    rq, rs = O.quant_fp8_per_token(a)
    assert torch.isnan(rs[M - 2]) and torch.isinf(rs[M - 1])
    assert torch.allclose(sc.cpu(), rs, rtol=0, atol=0, equal_nan=True)
    got, want = q.cpu().view(torch.uint8), rq.view(torch.uint8)
    # inf / inf is NaN on both sides; its sign bit is the platform's default NaN
    nan = (want & 0x7F) == 0x7F
    assert torch.equal((got & 0x7F)[nan], want[nan] & 0x7F)
    assert torch.equal(got[~nan], want[~nan])
