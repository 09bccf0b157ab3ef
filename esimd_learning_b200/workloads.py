"""Seeded synthetic inputs for the benchmark configurations of the FP8 path.

No dataset is involved: every tensor is drawn from the distributions the
configurations name, on the CPU with `torch.manual_seed(seed)`, then moved
to the requested device.

  config 0  GEMV M=1, N=K=4096, x ~ N(0,1) fp16, W ~ N(0, 0.02) quantised
            per output row to e4m3 with fp32 scale = rowabsmax / 448
  config 1  batched GEMV M in {1,2,4,8} at (N,K) = (28672,4096) gate_up,
            (4096,14336) down, (6144,4096) QKV
  config 2  add+RMSNorm (eps 1e-6, gamma = 1 + 0.1 N(0,1)) -> QKV GEMV [6144,4096]
  config 3  prefill GEMM: A [M,4096] ~ N(0,1) per-token quantised, B [14336,4096]
  config 4  70B-shaped decode chain, hidden 8192 (see esimd_learning_b200.chain)
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0

CONFIG1_SHAPES = {"gate_up": (28672, 4096), "down": (4096, 14336), "qkv": (6144, 4096)}
CONFIG1_MS = (1, 2, 4, 8)


def quantize_per_channel(w: torch.Tensor, fp8_dtype=torch.float8_e4m3fn):
    """Per-output-row FP8 quantisation: scale = rowabsmax / fmax (fp32 [N]),
    wq = fp8(clamp(w / scale, -fmax, fmax))."""
    fmax = torch.finfo(fp8_dtype).max
    wf = w.float()
    scale = wf.abs().amax(dim=1).clamp(min=1e-12) / fmax
    wq = (wf / scale[:, None]).clamp(-fmax, fmax).to(fp8_dtype)
    return wq, scale


def make_fp8_weight(N: int, K: int, gen: torch.Generator, std: float = 0.02,
                    fp8_dtype=torch.float8_e4m3fn):
    w = torch.randn(N, K, generator=gen, dtype=torch.float32) * std
    return quantize_per_channel(w, fp8_dtype)


def gemv_case(M: int, N: int, K: int, seed: int = 0, dtype=torch.float16, device="cpu"):
    """(x [M,K], wq [N,K] e4m3, scale fp32 [N]) per config 0/1."""
    gen = torch.Generator().manual_seed(seed)
    wq, scale = make_fp8_weight(N, K, gen)
    x = torch.randn(M, K, generator=gen, dtype=torch.float32).to(dtype)
    return x.to(device), wq.to(device), scale.to(device)


def fused_norm_case(M: int, N: int = 6144, K: int = 4096, seed: int = 0, dtype=torch.float16,
                    device="cpu"):
    """(hidden, residual, gamma, wq, scale) per config 2."""
    gen = torch.Generator().manual_seed(seed)
    hidden = torch.randn(M, K, generator=gen).to(dtype)
    residual = torch.randn(M, K, generator=gen).to(dtype)
    gamma = (1.0 + 0.1 * torch.randn(K, generator=gen)).to(dtype)
    wq, scale = make_fp8_weight(N, K, gen)
    return tuple(t.to(device) for t in (hidden, residual, gamma, wq, scale))


def prefill_case(M: int, N: int = 14336, K: int = 4096, seed: int = 0, dtype=torch.float16,
                 device="cpu"):
    """(A [M,K] io dtype, bq [N,K] e4m3, b_scale fp32 [N]) per config 3."""
    gen = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=gen).to(dtype)
    bq, bs = make_fp8_weight(N, K, gen)
    return a.to(device), bq.to(device), bs.to(device)
