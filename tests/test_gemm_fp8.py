"""FP8 GEMM on the GPU against the oracle.

* esimd_gemm_fp8_pert (the reference op): the reference's
  tests/test_gemm_fp8.py shapes, M in {1..64}, fp16/bf16 I/O, e4m3/e5m2
  weights, and GEMM(M=1) == GEMV (tests/test_gemm_fp8.py:65-93).
* esimd_gemm_fp8_pert at prefill sizes (M > 64): the weight dequantised to
  fp16/bf16, then the kind::f16 tcgen05 GEMM; ragged M, N tails, and the C ABI
  with a per-N scale.
* the tcgen05 prefill GEMM (per-token x per-channel scales)
  shapes and ragged M / N edges, against the fp32 oracle of the same
  quantised operands; quantisation itself is bit-exact (test_elementwise).
"""
from pathlib import Path

import pytest
import torch

from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import prefill_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF_SHAPES = [(2560, 2048), (512, 2048), (2048, 512), (128, 2048), (3072, 2048), (1024, 1024)]
REF_MS = [1, 2, 4, 8, 16, 32, 64]


@pytest.mark.parametrize("N,K", REF_SHAPES)
@pytest.mark.parametrize("wdt", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_gemm_pert_correctness(ext, cuda_device, N, K, wdt, io):
    torch.manual_seed(0)
    for M in REF_MS:
        w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(wdt)
        sv = 0.05 + torch.rand(1).item() * 0.1
        x = (torch.randn(M, K) * 0.1).to(io)
        out = torch.zeros(M, N, dtype=io, device=cuda_device)
        ext.esimd_gemm_fp8_pert(x.to(cuda_device), w.to(cuda_device),
                                torch.tensor(sv, dtype=torch.float32, device=cuda_device), out)
        O.assert_parity(out, O.gemv_fp8(x, w, torch.tensor(sv)), f"M={M} N={N} K={K} {wdt} {io}")


@pytest.mark.parametrize("M,N,K", [(65, 256, 512), (128, 512, 256), (300, 1040, 384), (257, 2048, 2048),
                                   (1000, 4096, 1024),
                                   # either side of cek_gemm_fp8w_preferred's crossovers
                                   (25, 14336, 4096), (26, 14336, 4096), (111, 4096, 14336), (112, 4096, 14336)])
@pytest.mark.parametrize("wdt", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_gemm_pert_prefill(ext, cuda_device, M, N, K, wdt, io):
    torch.manual_seed(1)
    w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(wdt)
    sv = 0.05 + torch.rand(1).item() * 0.1
    x = (torch.randn(M, K) * 0.1).to(io)
    out = torch.full((M, N), float("nan"), dtype=io, device=cuda_device)
    ext.esimd_gemm_fp8_pert(x.to(cuda_device), w.to(cuda_device),
                            torch.tensor(sv, dtype=torch.float32, device=cuda_device), out)
    O.assert_parity(out, O.gemv_fp8(x, w, torch.tensor(sv)), f"M={M} N={N} K={K} {wdt} {io}")


def test_gemm_pert_prefill_config3(ext, cuda_device):
    """fp16 activations [2048, 4096] x e4m3 [14336, 4096], per-tensor scale;
    the oracle checks a strided sample of rows."""
    M, N, K = 2048, 14336, 4096
    torch.manual_seed(2)
    w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(torch.float8_e4m3fn)
    x = (torch.randn(M, K) * 0.1).half()
    s = torch.tensor(0.07, dtype=torch.float32)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    ext.esimd_gemm_fp8_pert(x.to(cuda_device), w.to(cuda_device), s.to(cuda_device), out)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    rows = torch.arange(0, M, 67)
    O.assert_parity(out.cpu()[rows], O.gemv_fp8(x[rows], w, s), "pert prefill config3")


def test_gemm_fp8w_cabi_pern(cuda_device):
    """C ABI with a per-N fp32 scale, bf16 I/O, e4m3 and e5m2 weights, at a
    small M (weight tiles converted in shared memory) and a large one
    (dequantised into the workspace first); workspace size rule; shape
    checks."""
    N, K = 272, 320
    torch.manual_seed(3)
    L = cabi.lib()
    nb = L.cek_gemm_fp8w_workspace_bytes(N, K)
    assert nb >= N * K * 2 and nb % 256 == 0
    ws = torch.empty(nb, dtype=torch.uint8, device=cuda_device)
    for M, wdt in ((200, torch.float8_e4m3fn), (200, torch.float8_e5m2), (300, torch.float8_e5m2)):
        w = (torch.randn(N, K, dtype=torch.float16) * 0.1).to(wdt)
        sc = torch.rand(N) * 0.1 + 0.01
        x = (torch.randn(M, K) * 0.1).bfloat16()
        wd, sd, xd = w.to(cuda_device), sc.to(cuda_device), x.to(cuda_device)
        y = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda_device)
        cabi.call("cek_gemm_fp8w", cabi.ptr(xd), cabi.ptr(wd), cabi.ptr(sd), cabi.ptr(y), cabi.ptr(ws), nb,
                  M, N, K, cabi.CEK_BF16, cabi.fp8_format(wd), cabi.CEK_SCALE_PERN_F32, cabi.current_stream())
        torch.cuda.synchronize()
        O.assert_parity(y, O.gemv_fp8(x, w, sc), f"fp8w cabi pern M={M} {wdt}")
    args = (cabi.ptr(xd), cabi.ptr(wd), cabi.ptr(sd), cabi.ptr(y), cabi.ptr(ws), nb)
    assert L.cek_gemm_fp8w(cabi.ptr(xd), cabi.ptr(wd), cabi.ptr(sd), cabi.ptr(y), cabi.ptr(ws), nb - 256, M, N, K,
                           cabi.CEK_BF16, cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_gemm_fp8w(*args, M, N, 96, cabi.CEK_BF16, cabi.CEK_E4M3,
                           cabi.CEK_SCALE_PERN_F32, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_gemm_fp8w(*args, M, 250, K, cabi.CEK_BF16, cabi.CEK_E4M3,
                           cabi.CEK_SCALE_PERN_F32, None) == cabi.CEK_ERR_INVALID_ARG
    n = __import__("ctypes").c_uint64(99)
    cabi.call("cek_gemm_fp8_timeouts", __import__("ctypes").byref(n))
    assert n.value == 0


def test_gemm_vs_gemv_m1(ext, cuda_device):
    for io in (torch.float16, torch.bfloat16):
        for N, K in [(2560, 2048), (512, 2048), (128, 2048), (2048, 512)]:
            w = (torch.randn(N, K, dtype=torch.float16, device=cuda_device) * 0.1).to(torch.float8_e4m3fn)
            s = torch.tensor(0.073, dtype=torch.float32, device=cuda_device)
            x = (torch.randn(1, K, device=cuda_device) * 0.1).to(io)
            a = torch.zeros(1, N, dtype=io, device=cuda_device)
            b = torch.zeros(1, N, dtype=io, device=cuda_device)
            ext.esimd_gemv_fp8_pert(x, w, s, a)
            ext.esimd_gemm_fp8_pert(x, w, s, b)
            rel = (a.float() - b.float()).abs().max().item() / a.float().abs().max().item()
            assert rel < 0.01


def _prefill(ext, dev, M, N, K, io=torch.float16, seed=0):
    a, bq, bs = prefill_case(M, N=N, K=K, seed=seed, dtype=io)
    aq, as_ = O.quant_fp8_per_token(a)
    y = torch.full((M, N), float("nan"), dtype=io, device=dev)
    ext.esimd_gemm_fp8_pertoken_pern(aq.to(dev), as_.to(dev), bq.to(dev), bs.to(dev), y)
    torch.cuda.synchronize()
    return y, O.gemm_fp8_scaled(aq, as_, bq, bs, out_dtype=io)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 512), (100, 272, 256), (300, 1040, 384), (640, 2240, 256), (130, 3840, 128),
                                   (1, 16, 128), (129, 4096, 1024)])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_tcgen05_gemm_small(ext, cuda_device, M, N, K, io):
    y, ref = _prefill(ext, cuda_device, M, N, K, io)
    O.assert_parity(y, ref, f"M={M} N={N} K={K}")


@pytest.mark.parametrize("M", [2048, 8192])
def test_tcgen05_gemm_config3(ext, cuda_device, M):
    """A [M, 4096] per-token e4m3, B [14336, 4096] per-channel e4m3.
    The oracle runs on the rows of a strided sample (full fp32 CPU GEMM at M=8192
    would take minutes); every row of the GPU output is checked finite."""
    N, K = 14336, 4096
    a, bq, bs = prefill_case(M, N=N, K=K, seed=0)
    dev = cuda_device
    ad = a.to(dev)
    aq = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=dev)
    as_ = torch.empty(M, dtype=torch.float32, device=dev)
    ext.esimd_quant_fp8_per_token(ad, aq, as_)
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    ext.esimd_gemm_fp8_pertoken_pern(aq, as_, bq.to(dev), bs.to(dev), y)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    rows = torch.arange(0, M, 61)
    ref = O.gemm_fp8_scaled(aq.cpu()[rows], as_.cpu()[rows], bq, bs)
    O.assert_parity(y.cpu()[rows], ref, f"config3 M={M}")
    # fp16 reference semantics end to end: quantised GEMM vs the unquantised product
    full = (a[rows].float() @ (bq.float() * bs[:, None]).T)
    m = O.parity(y.cpu()[rows], full)
    assert m["mean_rel"] < 0.05
    # every row: the oracle's formula in plain fp32 torch on the GPU (exact
    # FP8 -> fp32 decode from the oracle's table, true fp32 matmul, no TF32),
    # itself pinned to the CPU oracle on the sampled rows above
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        af = O.fp8_decode(aq.cpu(), O.E4M3).reshape(M, K).to(dev)
        bf = O.fp8_decode(bq, O.E4M3).reshape(N, K).to(dev)
        ref_all = ((af @ bf.T) * as_.reshape(-1, 1) * bs.to(dev).reshape(1, -1)).half()
        del af, bf
        O.assert_parity(ref_all[rows].cpu(), ref, f"fp32 GPU reference vs CPU oracle M={M}")
        for r0 in range(0, M, 1024):  # every row, in blocks (the metric is per block)
            O.assert_parity(y[r0:r0 + 1024], ref_all[r0:r0 + 1024], f"config3 M={M} rows {r0}..")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32


def test_tcgen05_gemm_cabi_and_timeouts(cuda_device):
    M, N, K = 256, 512, 256
    a, bq, bs = prefill_case(M, N=N, K=K, seed=3, device=cuda_device)
    aq, as_ = O.quant_fp8_per_token(a.cpu())
    aq, as_ = aq.to(cuda_device), as_.to(cuda_device)
    y = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda_device)
    cabi.call("cek_gemm_fp8_scaled", cabi.ptr(aq), cabi.ptr(bq), cabi.ptr(as_), cabi.ptr(bs), cabi.ptr(y),
              M, N, K, cabi.CEK_BF16, cabi.current_stream())
    torch.cuda.synchronize()
    O.assert_parity(y, O.gemm_fp8_scaled(aq.cpu(), as_.cpu(), bq.cpu(), bs.cpu(), out_dtype=torch.bfloat16),
                    "cabi")
    import ctypes
    n = ctypes.c_uint64(99)
    cabi.call("cek_gemm_fp8_timeouts", ctypes.byref(n))
    assert n.value == 0


def test_tcgen05_gemm_rejects_bad_shapes(cuda_device):
    L = cabi.lib()
    assert L.cek_gemm_fp8_scaled(16, 16, 16, 16, 16, 128, 256, 100, 0, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_gemm_fp8_scaled(16, 16, 16, 16, 16, 128, 250, 128, 0, None) == cabi.CEK_ERR_INVALID_ARG


def test_tcgen05_gemm_cta_pair_path(cuda_device):
    """The CTA-pair variant of the per-token FP8 GEMM (tcgen05 cta_group::2,
    cluster of 2, enabled by CEK_GEMM_PAIR=1) against the oracle, in a child
    process (the switch is read once per process): ragged M and N edges, and
    the config-3 shape."""
    import os
    import subprocess
    import sys
    code = r'''
import sys, ctypes, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/python")
import esimd_learning_b200 as ops
from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import prefill_case
from oracle import oracle as O
dev = torch.device("cuda", 0)
for M, N, K in [(256, 512, 256), (300, 1040, 512), (1000, 2048, 1024), (2048, 14336, 4096)]:
    a, bq, bs = prefill_case(M, N=N, K=K, seed=M)
    aq, as_ = O.quant_fp8_per_token(a)
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
    ops.esimd_gemm_fp8_pertoken_pern(aq.to(dev), as_.to(dev), bq.to(dev), bs.to(dev), y)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all(), (M, N, K)
    rows = torch.arange(0, M, max(1, M // 61))
    O.assert_parity(y.cpu()[rows], O.gemm_fp8_scaled(aq[rows], as_[rows], bq, bs), f"pair M={M} N={N} K={K}")
n = ctypes.c_uint64(1); cabi.call("cek_gemm_fp8_timeouts", ctypes.byref(n)); assert n.value == 0
print("pair ok")
'''
    root = str(Path(__file__).resolve().parent.parent)
    r = subprocess.run([sys.executable, "-c", code, root], capture_output=True, text=True, timeout=600,
                       env={**os.environ, "CEK_GEMM_PAIR": "1"})
    assert r.returncode == 0 and "pair ok" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]
