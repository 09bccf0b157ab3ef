"""B200 (sm_100a) FP8 custom-op package: a drop-in for the reference's
`custom_esimd_kernels_vllm` Python package
(python/custom_esimd_kernels_vllm/__init__.py:1-13).

Importing it loads the two torch.library extension modules, which register
the ops in the `torch.ops.custom_esimd_kernels_vllm` namespace on the CUDA
dispatch key, and re-exports the Python wrappers of `ops`.  A vLLM build that
calls `torch.ops.custom_esimd_kernels_vllm.*` or `from custom_esimd_kernels_vllm
import ...` can point at this package instead (`import esimd_learning_b200 as
custom_esimd_kernels_vllm`).

There is no CPU or eager fallback: if the extensions were not built the import
fails with the command that builds them.
"""
import torch  # noqa: F401  (loads libtorch before the extension modules)

try:
    from esimd_learning_b200 import custom_esimd_kernels  # noqa: F401
    from esimd_learning_b200 import custom_esimd_kernels_gemm  # noqa: F401
except ImportError as e:  # pragma: no cover - exercised only on an unbuilt tree
    raise ImportError(
        "esimd_learning_b200 extensions are not built; run "
        "`python esimd_learning_b200/build.py` (needs nvcc with sm_100a support)"
    ) from e

from esimd_learning_b200.ops import (  # noqa: E402,F401
    esimd_gemv_fp8_pern,
    esimd_gemv_fp8_pert,
    esimd_gemv_fp8_pern_fused,
    esimd_fused_add_rms_norm_batched,
    esimd_gemm_fp8_pert,
    esimd_fused_add_rms_norm_batched_fp8,
    esimd_gelu_and_mul,
    esimd_gemv_fp8_gelu_mul,
    esimd_fused_add_rms_norm_gelu_mul_fp8,
    esimd_qkv_norm_rope,
    esimd_quant_fp8_per_token,
    esimd_set_weight_prefetch,
    esimd_gemm_fp8_pertoken_pern,
)
