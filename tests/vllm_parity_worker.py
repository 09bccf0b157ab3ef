"""Child process of tests/test_vllm_parity.py: runs this build's decode-helper
ops and vLLM's published CUDA implementations of the same operations on the
same seeded inputs, and prints one JSON line of agreement metrics.  vLLM is
imported only here, so its import and kernels cannot affect the test process."""
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "python"))
sys.path.insert(0, str(ROOT))

import esimd_learning_b200 as ops  # noqa: E402
from oracle import oracle as O  # noqa: E402


def ulp_stats(a: torch.Tensor, b: torch.Tensor) -> dict:
    """Agreement of two fp16/bf16 tensors: fraction of differing elements and
    the largest difference in units of the last place of the larger value."""
    af, bf = a.float(), b.float()
    diff = (af - bf).abs()
    mag = torch.maximum(af.abs(), bf.abs())
    mant = 10 if a.dtype == torch.float16 else 7
    ulp = torch.exp2(torch.floor(torch.log2(mag.clamp(min=2.0 ** -14))) - mant)
    return {"frac_diff": (diff > 0).float().mean().item(), "max_ulp": (diff / ulp).max().item()}


def main():
    import vllm
    from vllm import _custom_ops as vops  # registers torch.ops._C
    dev = torch.device("cuda", 0)
    res = {"vllm": vllm.__version__}
    g = torch.Generator(device=dev).manual_seed(0)

    # GeLU(tanh)-and-mul: vLLM gelu_tanh_and_mul (gate first half, up second)
    for io in (torch.float16, torch.bfloat16):
        for M, d in ((1, 28672), (16, 3584)):
            x = (torch.randn(M, 2 * d, device=dev, generator=g) * 2).to(io)
            ours = torch.empty(M, d, dtype=io, device=dev)
            ops.esimd_gelu_and_mul(x, ours)
            theirs = torch.empty(M, d, dtype=io, device=dev)
            torch.ops._C.gelu_tanh_and_mul(theirs, x)
            # error of each against the float64 value of the same formula
            xd = x.double()
            gd, ud = xd[:, :d], xd[:, d:]
            exact = 0.5 * gd * (1 + torch.tanh((2 / torch.pi) ** 0.5 * (gd + 0.044715 * gd ** 3))) * ud
            res[f"gelu_{str(io)[6:]}_M{M}"] = {
                **ulp_stats(ours, theirs),
                "ours_mean_abs_err": (ours.double() - exact).abs().mean().item(),
                "vllm_mean_abs_err": (theirs.double() - exact).abs().mean().item()}

    # q/k per-head RMSNorm + RoPE (neox, theta 500000): vLLM rms_norm on each
    # head, then rotary_embedding with the same cos | sin cache
    hq, hkv, D, eps = 64, 8, 128, 1e-6
    cs = O.rope_cos_sin_cache(8192, D, 500000.0).to(dev)
    for io in (torch.float16, torch.bfloat16):
        M = 8
        qkv = torch.randn(M, (hq + 2 * hkv) * D, device=dev, generator=g).to(io)
        pos = torch.randint(0, 8192, (M,), device=dev, generator=g)
        qw = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(io)
        kw = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(io)
        ours = qkv.clone()
        ops.esimd_qkv_norm_rope(ours, pos, qw, kw, cs, hq, hkv, D, eps, True)
        q_in = qkv[:, : hq * D].reshape(M * hq, D).contiguous()
        k_in = qkv[:, hq * D:(hq + hkv) * D].reshape(M * hkv, D).contiguous()
        q = torch.empty_like(q_in)
        k = torch.empty_like(k_in)
        torch.ops._C.rms_norm(q, q_in, qw, eps)
        torch.ops._C.rms_norm(k, k_in, kw, eps)
        q, k = q.reshape(M, hq * D), k.reshape(M, hkv * D)
        try:
            torch.ops._C.rotary_embedding(pos, q, k, D, cs, True)
            cache = "fp32"
        except RuntimeError:
            torch.ops._C.rotary_embedding(pos, q, k, D, cs.to(io), True)
            cache = str(io)
        theirs = torch.cat([q, k], dim=1)
        key = f"qkv_norm_rope_{str(io)[6:]}"
        res[key] = {**ulp_stats(ours[:, :(hq + hkv) * D], theirs), "vllm_cache": cache,
                    **O.parity(ours[:, :(hq + hkv) * D], theirs)}
        res[key]["v_untouched"] = bool(torch.equal(ours[:, (hq + hkv) * D:], qkv[:, (hq + hkv) * D:]))

    # per-token dynamic e4m3 quantisation: vLLM scaled_fp8_quant(per token)
    for io in (torch.float16, torch.bfloat16):
        M, K = 2048, 4096
        a = torch.randn(M, K, device=dev, generator=g).to(io)
        q = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty(M, dtype=torch.float32, device=dev)
        ops.esimd_quant_fp8_per_token(a, q, s)
        vq, vs = vops.scaled_fp8_quant(a, use_per_token_if_dynamic=True)
        vs = vs.reshape(-1)
        co = q.view(torch.uint8).int()
        cv = vq.view(torch.uint8).int()
        res[f"quant_{str(io)[6:]}"] = {
            "scale_max_rel": ((s - vs).abs() / vs.abs()).max().item(),
            "codes_frac_diff": (co != cv).float().mean().item(),
            # e4m3 magnitudes are monotonic in the low 7 code bits: 1 = one representable step
            "codes_max_step": ((co & 0x7F) - (cv & 0x7F)).abs().max().item(),
            "sign_mismatch": int(((((co ^ cv) & 0x80) != 0) & (((co & 0x7F) + (cv & 0x7F)) > 0)).sum().item()),
            **{f"deq_{k}": v for k, v in O.parity(q.float() * s[:, None], vq.float() * vs[:, None]).items()},
        }
    print(json.dumps(res))


if __name__ == "__main__":
    main()
