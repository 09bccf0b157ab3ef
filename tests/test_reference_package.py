"""The reference's own import line works unchanged:
`from custom_esimd_kernels_vllm import ...` (python/custom_esimd_kernels_vllm/
__init__.py:1-13) loads this build's extension modules and wrappers, and each
of the four reference ops matches the oracle through that import.

The CPU test checks the package layout (submodule names, wrapper names); the
GPU test calls each op once, as the reference tests do
(tests/test_gemv_fp8.py, test_gemm_fp8.py, test_fused_add_rms_norm_batched_fp8.py).
"""
import importlib

import pytest
import torch

from oracle import oracle as O


def test_reference_import_line_resolves():
    pkg = importlib.import_module("custom_esimd_kernels_vllm")
    assert pkg.__file__.replace("\\", "/").endswith("python/custom_esimd_kernels_vllm/__init__.py")
    for sub in ("custom_esimd_kernels", "custom_esimd_kernels_gemm", "ops"):
        assert importlib.import_module(f"custom_esimd_kernels_vllm.{sub}") is not None
    from custom_esimd_kernels_vllm import (esimd_fused_add_rms_norm_batched, esimd_gemm_fp8_pert,  # noqa: F401
                                           esimd_gemv_fp8_pern, esimd_gemv_fp8_pert)
    import esimd_learning_b200
    assert esimd_learning_b200.esimd_gemv_fp8_pern is pkg.esimd_gemv_fp8_pern


@pytest.mark.gpu
def test_reference_ops_through_reference_package(cuda_device):
    from custom_esimd_kernels_vllm import (esimd_fused_add_rms_norm_batched, esimd_gemm_fp8_pert,
                                           esimd_gemv_fp8_pern, esimd_gemv_fp8_pert)
    from esimd_learning_b200.workloads import gemv_case
    dev = cuda_device
    N, K = 4096, 4096
    x, wq, s = gemv_case(1, N, K, seed=0)
    # per-N scale as the reference passes it: fp16 [N]
    s16 = s.to(torch.float16)
    y = torch.zeros(1, N, dtype=torch.float16, device=dev)
    ret = esimd_gemv_fp8_pern(x.to(dev), wq.to(dev), s16.to(dev), y, N, K)
    assert ret.data_ptr() == y.data_ptr()
    O.assert_parity(y, O.gemv_fp8(x, wq, s16), "pern via custom_esimd_kernels_vllm")

    st = torch.tensor(0.0123, dtype=torch.float32)
    y = torch.zeros(1, N, dtype=torch.float16, device=dev)
    esimd_gemv_fp8_pert(x.to(dev), wq.to(dev), st.to(dev), y)
    O.assert_parity(y, O.gemv_fp8(x, wq, st), "pert via custom_esimd_kernels_vllm")

    for M in (4, 96):
        xm = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half()
        y = torch.zeros(M, N, dtype=torch.float16, device=dev)
        esimd_gemm_fp8_pert(xm.to(dev), wq.to(dev), st.to(dev), y)
        O.assert_parity(y, O.gemv_fp8(xm, wq, st), f"gemm pert M={M} via custom_esimd_kernels_vllm")

    g = torch.Generator().manual_seed(5)
    h = torch.randn(4, K, generator=g).half()
    r = torch.randn(4, K, generator=g).half()
    w = (1 + 0.1 * torch.randn(K, generator=g)).half()
    hd, rd = h.to(dev), r.to(dev)
    out = esimd_fused_add_rms_norm_batched(hd, rd, w.to(dev), 1e-6)
    assert out.data_ptr() == hd.data_ptr()
    ref_r, ref_h = O.add_rmsnorm(h, r, w, 1e-6)
    assert torch.equal(rd.cpu(), ref_r)
    O.assert_parity(hd, ref_h, "add+rmsnorm via custom_esimd_kernels_vllm")
