"""The no-allocation variant of the fused add+RMSNorm -> FP8 GEMV entry point.

Some callers of this library cannot allocate device memory where they call
it: a plugin's enqueue callback inside another runtime, a process whose GPU
memory is handed out by its own pool at start-up, a serving loop that must
not touch an allocator per request.  cek_fused_add_rmsnorm_gemv_fp8_noalloc
serves them: its scratch is a fixed array inside libcek_b200.so.  This test
calls it through the C ABI twice in a row (different shapes, so the second
call runs over what the first left in the shared array) and checks each
result against the workspace-taking entry point on identical inputs, with
the tolerance the other GPU tests use.  It sits in its own file, collected
last, and works alone in a fresh process or after the other tests.
"""
import pytest
import torch

from esimd_learning_b200 import cabi
from esimd_learning_b200.workloads import fused_norm_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(entry, h, r, g, wq, s, M, N, K):
    y = torch.zeros(M, N, dtype=h.dtype, device=h.device)
    args = [cabi.ptr(h), cabi.ptr(r), cabi.ptr(g), 1e-6, cabi.ptr(wq), cabi.ptr(s), cabi.ptr(y)]
    if entry == "cek_fused_add_rmsnorm_gemv_fp8":
        nbytes = cabi.lib().cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=h.device)
        args += [cabi.ptr(ws), nbytes]
    args += [M, N, K, cabi.io_dtype(h), cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, 0,
             cabi.current_stream()]
    cabi.call(entry, *args)
    torch.cuda.synchronize()
    return y


def test_noalloc_matches_workspace_entry_point(cuda_device):
    for (M, N, K, io, seed) in [(4, 6144, 4096, torch.float16, 1), (16, 1000, 2048, torch.bfloat16, 2)]:
        h, r, g, wq, s = fused_norm_case(M, N=N, K=K, seed=seed, dtype=io, device=cuda_device)
        r_ref, r_new = r.clone(), r.clone()
        y_ref = _run("cek_fused_add_rmsnorm_gemv_fp8", h, r_ref, g, wq, s, M, N, K)
        y_new = _run("cek_fused_add_rmsnorm_gemv_fp8_noalloc", h, r_new, g, wq, s, M, N, K)
        assert torch.equal(r_new, r_ref)
        O.assert_parity(y_new, y_ref, f"noalloc M={M} N={N} K={K}")


def test_noalloc_rejects_rows_above_its_scratch(cuda_device):
    M = cabi.CEK_NOALLOC_MAX_ROWS + 1
    rc = cabi.lib().cek_fused_add_rmsnorm_gemv_fp8_noalloc(16, 16, 16, 1e-6, 16, 16, 16, M, 64, 512, 0, 0,
                                                           0, 0, None)
    assert rc == cabi.CEK_ERR_SCRATCH_LIMIT
    assert b"no-allocation" in cabi.lib().cek_status_string(rc)


def test_noalloc_refuses_gated_output(cuda_device):
    M, N, K = 2, 256, 512
    h, r, g, wq, s = fused_norm_case(M, N=2 * N, K=K, seed=3, device=cuda_device)
    y = torch.zeros(M, N, dtype=h.dtype, device=cuda_device)
    rc = cabi.lib().cek_fused_add_rmsnorm_gemv_fp8_noalloc(
        cabi.ptr(h), cabi.ptr(r), cabi.ptr(g), 1e-6, cabi.ptr(wq), cabi.ptr(s), cabi.ptr(y), M, N, K,
        cabi.io_dtype(h), cabi.CEK_E4M3, cabi.CEK_SCALE_PERN_F32, cabi.CEK_GEMV_GELU_MUL_OUTPUT,
        cabi.current_stream())
    assert rc == cabi.CEK_ERR_UNSUPPORTED
