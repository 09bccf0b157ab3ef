"""B200 (sm_100a) implementation of the FP8 custom-op path.

The kernels are in `libcek_b200.so` (C ABI: include/cek.h); the torch.library
registration and the Python wrappers are the package `custom_esimd_kernels_vllm`
(under `python/`, the reference's name and layout).  Importing this package
puts `python/` on the import path, loads that wrapper package and re-exports
its ops, so `import esimd_learning_b200 as ops; ops.esimd_gemv_fp8_pern(...)`
and `from custom_esimd_kernels_vllm import esimd_gemv_fp8_pern` reach the same
op.  The decode-chain driver (`chain`), the C-ABI loader (`cabi`) and the
vLLM linear method (`vllm_linear`) live here.
"""
import sys
from pathlib import Path

_PY = str(Path(__file__).resolve().parent.parent / "python")
if _PY not in sys.path:
    sys.path.insert(0, _PY)

import custom_esimd_kernels_vllm  # noqa: E402,F401
from custom_esimd_kernels_vllm import ops  # noqa: E402,F401
from custom_esimd_kernels_vllm.ops import (  # noqa: E402,F401
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
