"""Registers this package's W8A16 FP8 linear method with vLLM as the
quantization method ``"esimd_fp8"`` (vLLM 0.22 ``register_quantization_config``),
so that a vLLM model whose config names it builds its linear layers on the
esimd kernels: the same routing the reference's ops give vLLM on XPU
(tests/test_gemv_fp8.py:254-279 compares them with vLLM's
``fp8_gemm_w8a16``).

Call ``register()`` once before building the model.  vLLM is imported only
inside it; nothing else in the package needs vLLM.
"""
from __future__ import annotations

import torch

from esimd_learning_b200.vllm_linear import EsimdFp8LinearMethod

NAME = "esimd_fp8"
_registered = None


def register(name: str = NAME):
    """Registers (once) and returns the QuantizationConfig class."""
    global _registered
    if _registered is not None:
        return _registered
    from vllm.model_executor.layers.linear import LinearBase, LinearMethodBase
    from vllm.model_executor.layers.quantization import register_quantization_config
    from vllm.model_executor.layers.quantization.base_config import QuantizationConfig
    from vllm.model_executor.utils import set_weight_attrs

    class EsimdFp8VllmLinearMethod(LinearMethodBase):
        """vLLM LinearMethodBase over EsimdFp8LinearMethod: weight [N, K]
        float8 with a per-channel (or per-tensor) fp32 weight_scale, loaded by
        the layer's own weight_loader, fp16/bf16 activations."""

        def __init__(self, config: "EsimdFp8Config"):
            self.config = config
            self.impl = EsimdFp8LinearMethod(config.fp8_dtype)

        def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                           params_dtype, **extra_weight_attrs):
            self.impl.create_weights(layer, input_size_per_partition, output_partition_sizes, input_size,
                                     output_size, params_dtype, per_tensor=self.config.per_tensor)
            set_weight_attrs(layer.weight, {"input_dim": 1, "output_dim": 0, **extra_weight_attrs})
            scale_attrs = dict(extra_weight_attrs)
            if not self.config.per_tensor:
                scale_attrs["output_dim"] = 0
            set_weight_attrs(layer.weight_scale, scale_attrs)

        def process_weights_after_loading(self, layer) -> None:
            self.impl.process_weights_after_loading(layer)

        def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
            return self.impl.apply(layer, x, bias)

    @register_quantization_config(name)
    class EsimdFp8Config(QuantizationConfig):
        """FP8 weight-only (W8A16) checkpoints run on the esimd B200 kernels."""

        def __init__(self, fp8_dtype=torch.float8_e4m3fn, per_tensor: bool = False):
            super().__init__()
            self.fp8_dtype = fp8_dtype
            self.per_tensor = per_tensor

        def get_name(self) -> str:
            return name

        def get_supported_act_dtypes(self) -> list[torch.dtype]:
            return [torch.float16, torch.bfloat16]

        @classmethod
        def get_min_capability(cls) -> int:
            return 100  # sm_100a kernels

        @staticmethod
        def get_config_filenames() -> list[str]:
            return []

        @classmethod
        def from_config(cls, config: dict) -> "EsimdFp8Config":
            fmt = str(config.get("fmt", "e4m3"))
            return cls(torch.float8_e5m2 if fmt == "e5m2" else torch.float8_e4m3fn,
                       bool(config.get("per_tensor", False)))

        def get_quant_method(self, layer: torch.nn.Module, prefix: str):
            return EsimdFp8VllmLinearMethod(self) if isinstance(layer, LinearBase) else None

    _registered = EsimdFp8Config
    return EsimdFp8Config
