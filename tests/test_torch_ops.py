"""torch.library boundary, no GPU: the ops exist under the reference's
namespace with the reference's schemas (csrc/xpu/torch_extension.cc:9-18,
torch_extension_gemm.cc:11-13) and fail loudly on non-CUDA tensors (there is
no CPU fallback)."""
import pytest
import torch

REFERENCE_SCHEMAS = {
    "esimd_gemv_fp8_pern": "esimd_gemv_fp8_pern(Tensor input, Tensor weight, Tensor weight_scale, "
                           "Tensor output, int N, int K) -> Tensor",
    "esimd_gemv_fp8_pert": "esimd_gemv_fp8_pert(Tensor input, Tensor weight, Tensor weight_scale, "
                           "Tensor output) -> Tensor",
    "esimd_fused_add_rms_norm_batched": "esimd_fused_add_rms_norm_batched(Tensor hidden_states, "
                                        "Tensor residual, Tensor weight, float eps) -> Tensor",
    "esimd_gemm_fp8_pert": "esimd_gemm_fp8_pert(Tensor input, Tensor weight, Tensor weight_scale, "
                           "Tensor output) -> Tensor",
}


def _schema(name):
    op = getattr(torch.ops.custom_esimd_kernels_vllm, name)
    return str(op.default._schema)


def test_reference_schemas_are_identical(ext):
    for name, schema in REFERENCE_SCHEMAS.items():
        assert _schema(name) == "custom_esimd_kernels_vllm::" + schema


def test_new_ops_registered(ext):
    for name in ("esimd_fused_add_rms_norm_batched_fp8", "esimd_gelu_and_mul",
                 "esimd_qkv_norm_rope", "esimd_quant_fp8_per_token", "esimd_set_weight_prefetch",
                 "esimd_gemv_fp8_pern_fused",
                 "esimd_gemm_fp8_pertoken_pern"):
        assert hasattr(torch.ops.custom_esimd_kernels_vllm, name)


def test_python_wrappers_mirror_reference_names(ext):
    for name in REFERENCE_SCHEMAS:
        assert callable(getattr(ext, name))


def test_cpu_tensors_fail_loudly(ext):
    x = torch.zeros(1, 64, dtype=torch.float16)
    w = torch.zeros(16, 64, dtype=torch.float8_e4m3fn)
    s = torch.ones(16, dtype=torch.float16)
    y = torch.zeros(1, 16, dtype=torch.float16)
    with pytest.raises(NotImplementedError):
        ext.esimd_gemv_fp8_pern(x, w, s, y, 16, 64)



def test_weight_prefetch_switch(ext):
    assert ext.esimd_set_weight_prefetch(True) is False
    assert ext.esimd_set_weight_prefetch(False) is True
