"""The vLLM custom-op wrapper package, under the reference's own name and
layout (python/custom_esimd_kernels_vllm/__init__.py:1-13), for NVIDIA B200.

Importing it loads its two torch.library extension modules, which register
the ops in the `torch.ops.custom_esimd_kernels_vllm` namespace on the CUDA
dispatch key (the kernels live in esimd_learning_b200/libcek_b200.so), and
re-exports the Python wrappers of `ops`.  A caller of the XPU build keeps its
imports unchanged:

    from custom_esimd_kernels_vllm import esimd_gemv_fp8_pern

There is no CPU or eager fallback: if the extensions were not built the import
fails with the command that builds them.
"""
import torch  # noqa: F401  (loads libtorch before the extension modules)

try:
    from custom_esimd_kernels_vllm import custom_esimd_kernels  # noqa: F401
    from custom_esimd_kernels_vllm import custom_esimd_kernels_gemm  # noqa: F401
except ImportError as e:  # pragma: no cover - exercised only on an unbuilt tree
    raise ImportError(
        "custom_esimd_kernels_vllm extensions are not built; run "
        "`python esimd_learning_b200/build.py` (needs nvcc with sm_100a support)"
    ) from e

from custom_esimd_kernels_vllm.ops import (  # noqa: E402,F401
    esimd_gemv_fp8_pern,
    esimd_gemv_fp8_pert,
    esimd_fused_add_rms_norm_batched,
    esimd_gemm_fp8_pert,
    esimd_gemv_fp8_pern_fused,
    esimd_fused_add_rms_norm_batched_fp8,
    esimd_gelu_and_mul,
    esimd_gemv_fp8_gelu_mul,
    esimd_fused_add_rms_norm_gelu_mul_fp8,
    esimd_qkv_norm_rope,
    esimd_quant_fp8_per_token,
    esimd_set_weight_prefetch,
    esimd_gemm_fp8_pertoken_pern,
)
