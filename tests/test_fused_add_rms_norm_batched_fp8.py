"""Residual add + RMSNorm (standalone, the reference op) and its fusion into
the FP8 GEMV, on the GPU against the oracle.

Mirrors tests/test_fused_add_rms_norm_batched_fp8.py of the reference
(K in {512, 1024, 2048, 4096}, M = 1, seed 42, its max < 0.1 check on the
normalised output) and adds the residual check it leaves commented out
(:51-54), bf16, batched rows, and BASELINE config 2.
"""
import pytest
import torch

from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import fused_norm_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_golden_vectors(ext, cuda_device, golden_cases):
    n = 0
    for c in golden_cases:
        if c["kind"] != "rmsnorm":
            continue
        h = c["hidden"].to(cuda_device)
        r = c["residual"].to(cuda_device)
        ext.esimd_fused_add_rms_norm_batched(h, r, c["weight"].to(cuda_device), c["eps"])
        assert (h.float().cpu() - c["ref_normed"]).abs().max().item() < 0.1  # reference bar
        O.assert_parity(h, c["ref_normed"], f"K={c['K']}")
        O.assert_parity(r, c["ref_residual"], f"residual K={c['K']}")
        n += 1
    assert n == 8


@pytest.mark.parametrize("K", [512, 1024, 2048, 4096, 8192, 16384, 8, 200])
@pytest.mark.parametrize("M", [1, 3, 8, 64])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_correctness_vs_oracle(ext, cuda_device, K, M, io):
    torch.manual_seed(42)
    h = torch.randn(M, K, dtype=io)
    r = torch.randn(M, K, dtype=io)
    w = (torch.randn(K) * 0.1 + 1.0).to(io)
    ref_r, ref_n = O.add_rmsnorm(h, r, w, 1e-6)
    hd, rd = h.to(cuda_device), r.to(cuda_device)
    out = ext.esimd_fused_add_rms_norm_batched(hd, rd, w.to(cuda_device), 1e-6)
    assert out.data_ptr() == hd.data_ptr()
    assert torch.equal(rd.cpu(), ref_r)  # residual add is exact up to the one rounding
    O.assert_parity(hd, ref_n, f"K={K} M={M}")


def test_zero_rows(ext, cuda_device):
    h = torch.zeros(0, 512, dtype=torch.float16, device=cuda_device)
    ext.esimd_fused_add_rms_norm_batched(h, h.clone(), torch.ones(512, dtype=torch.float16,
                                                                  device=cuda_device), 1e-6)


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_config2_fused_norm_gemv(ext, cuda_device, M, io):
    """add+RMSNorm (eps 1e-6, gamma = 1 + 0.1 N(0,1)) -> QKV [6144, 4096]."""
    h, r, g, wq, s = fused_norm_case(M, dtype=io)
    ref_r, ref_y = O.add_rmsnorm_gemv_fp8(h, r, g, 1e-6, wq, s)
    hd, rd = h.to(cuda_device), r.to(cuda_device)
    y = torch.zeros(M, 6144, dtype=io, device=cuda_device)
    ext.esimd_fused_add_rms_norm_batched_fp8(hd, rd, g.to(cuda_device), 1e-6, wq.to(cuda_device),
                                             s.to(cuda_device), y)
    assert torch.equal(hd.cpu(), h)  # hidden_states is only read
    assert torch.equal(rd.cpu(), ref_r)
    O.assert_parity(y, ref_y, f"config2 M={M}")


def test_fused_matches_unfused_composition(ext, cuda_device):
    """The fused op equals the reference's two ops run back to back."""
    h, r, g, wq, s = fused_norm_case(4, N=1024, K=2048, seed=3, device=cuda_device)
    h2, r2 = h.clone(), r.clone()
    y1 = torch.zeros(4, 1024, dtype=torch.float16, device=cuda_device)
    y2 = torch.zeros_like(y1)
    ext.esimd_fused_add_rms_norm_batched_fp8(h, r, g, 1e-6, wq, s, y1)
    ext.esimd_fused_add_rms_norm_batched(h2, r2, g, 1e-6)
    ext.esimd_gemv_fp8_pern(h2, wq, s, y2, 1024, 2048)
    torch.cuda.synchronize()
    assert torch.equal(r, r2)
    O.assert_parity(y1, y2.cpu(), "fused vs unfused")


def test_fused_through_cabi(cuda_device):
    h, r, g, wq, s = fused_norm_case(3, N=200, K=1024, seed=9, device=cuda_device)
    ref_r, ref_y = O.add_rmsnorm_gemv_fp8(h.cpu(), r.cpu(), g.cpu(), 1e-6, wq.cpu(), s.cpu())
    nbytes = cabi.lib().cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(3, 1024)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    y = torch.zeros(3, 200, dtype=torch.float16, device=cuda_device)
    cabi.call("cek_fused_add_rmsnorm_gemv_fp8", cabi.ptr(h), cabi.ptr(r), cabi.ptr(g), 1e-6,
              cabi.ptr(wq), cabi.ptr(s), cabi.ptr(y), cabi.ptr(ws), nbytes, 3, 200, 1024, cabi.CEK_F16,
              cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, 0, cabi.current_stream())
    torch.cuda.synchronize()
    assert torch.equal(r.cpu(), ref_r)
    O.assert_parity(y, ref_y, "cabi fused")


@pytest.mark.parametrize("io", [torch.float16, torch.bfloat16])
def test_fused_both_workspace_paths(cuda_device, io):
    """Full workspace: the normalised rows are staged for the GEMV; a 256-byte
    workspace: the GEMV forms them inside its loads.  Same residual, outputs
    within tolerance of each other and of the oracle."""
    M, N, K = 5, 3000, 4096
    h, r, g, wq, s = fused_norm_case(M, N=N, K=K, seed=13, dtype=io, device=cuda_device)
    ref_r, ref_y = O.add_rmsnorm_gemv_fp8(h.cpu(), r.cpu(), g.cpu(), 1e-6, wq.cpu(), s.cpu())
    outs = []
    for nbytes in (cabi.lib().cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K), 256):
        rr = r.clone()
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
        y = torch.zeros(M, N, dtype=io, device=cuda_device)
        cabi.call("cek_fused_add_rmsnorm_gemv_fp8", cabi.ptr(h), cabi.ptr(rr), cabi.ptr(g), 1e-6, cabi.ptr(wq),
                  cabi.ptr(s), cabi.ptr(y), cabi.ptr(ws), nbytes, M, N, K, cabi.io_dtype(h), cabi.CEK_E4M3,
                  cabi.CEK_SCALE_PERN_F32, 0, cabi.current_stream())
        torch.cuda.synchronize()
        assert torch.equal(rr.cpu(), ref_r)
        O.assert_parity(y, ref_y, f"workspace {nbytes}")
        outs.append(y)
    O.assert_parity(outs[0], outs[1].cpu(), "staged vs in-load")
