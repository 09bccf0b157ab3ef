"""An FP8 weight-only (W8A16) linear method on this package's kernels, shaped
like vLLM's ``LinearMethodBase`` (``create_weights`` /
``process_weights_after_loading`` / ``apply``), so that a vLLM CUDA build can
route its FP8 linear layers through the same ops the reference registers for
XPU.

vLLM stores an FP8 linear layer as ``weight`` [N, K] ``float8_e4m3fn`` (or
e5m2) with an fp32 ``weight_scale``, per output channel [N] or per tensor
[1].  ``apply`` keeps the activations in fp16/bf16, which is the reference
ops' arithmetic (no activation quantisation):

* few tokens (``cek_gemm_fp8w_preferred`` false: always for M <= 16, and
  up to M = 25 / 59 / 111 for 14336 x 4096 / 6144 x 4096 / 4096 x 14336):
  the GEMV family (``esimd_gemv_fp8_pern``, the bulk-copy kernel for
  M <= 16), one weight pass per 16-token tile;
* otherwise ``cek_gemm_fp8w``, a ``kind::f16`` tcgen05 GEMM on the weight
  converted exactly to 16 bits (in shared memory up to 256 tokens, into a
  workspace taken from the caching allocator for the call above), the
  scale in its epilogue.  K % 64 == 0 and N % 16 == 0 are needed; other
  shapes stay on the GEMV family.

``layer`` is any ``torch.nn.Module``; nothing here imports vLLM.
"""
from __future__ import annotations

import torch

GEMM_W8_MAX_TOKENS = 256  # CEK_GEMM_FP8W_INKERNEL_MAX_ROWS: no workspace up to this M


class EsimdFp8LinearMethod:
    """W8A16 FP8 linear layer: y = x @ deq(weight).T * weight_scale (+ bias)."""

    def __init__(self, fp8_dtype=torch.float8_e4m3fn):
        if fp8_dtype not in (torch.float8_e4m3fn, torch.float8_e5m2):
            raise ValueError("fp8_dtype must be float8_e4m3fn or float8_e5m2")
        self.fp8_dtype = fp8_dtype

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int,
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, per_tensor: bool = False, **extra) -> None:
        """Registers ``weight`` [sum(output_partition_sizes), K] and ``weight_scale``
        (fp32, [N] or [1]) on ``layer``, uninitialised, for the loader to fill."""
        n = sum(output_partition_sizes)
        k = input_size_per_partition
        layer.weight = torch.nn.Parameter(torch.empty(n, k, dtype=self.fp8_dtype), requires_grad=False)
        layer.weight_scale = torch.nn.Parameter(torch.empty(1 if per_tensor else n, dtype=torch.float32),
                                                requires_grad=False)
        layer.logical_widths = list(output_partition_sizes)
        layer.input_size_per_partition = k
        layer.output_size_per_partition = n
        layer.params_dtype = params_dtype

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        """Contiguous weight and an fp32 scale, as the kernels read them."""
        w = layer.weight.data
        if w.dtype not in (torch.float8_e4m3fn, torch.float8_e5m2) or w.dim() != 2:
            raise ValueError("weight must be a 2-D float8 tensor [N, K]")
        layer.weight = torch.nn.Parameter(w.contiguous(), requires_grad=False)
        s = layer.weight_scale.data.to(torch.float32).reshape(-1).contiguous()
        if s.numel() not in (1, w.shape[0]):
            raise ValueError("weight_scale must hold 1 or N values")
        layer.weight_scale = torch.nn.Parameter(s, requires_grad=False)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        import esimd_learning_b200 as ops
        from esimd_learning_b200 import cabi

        w, s = layer.weight, layer.weight_scale
        N, K = w.shape
        if x.shape[-1] != K:
            raise ValueError(f"input last dim {x.shape[-1]} != K {K}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, K).contiguous()
        M = x2.shape[0]
        y = torch.empty(M, N, dtype=x.dtype, device=x.device)
        if M == 0:
            return y.reshape(*lead, N)
        if cabi.lib().cek_gemm_fp8w_preferred(M, N, K):
            # the 16-bit weight copy is needed only above GEMM_W8_MAX_TOKENS
            nb = cabi.lib().cek_gemm_fp8w_workspace_bytes(N, K) if M > GEMM_W8_MAX_TOKENS else 0
            ws = torch.empty(nb, dtype=torch.uint8, device=x.device) if nb else None
            kind = cabi.CEK_SCALE_PERT_F32 if s.numel() == 1 else cabi.CEK_SCALE_PERN_F32
            cabi.call("cek_gemm_fp8w", cabi.ptr(x2), cabi.ptr(w), cabi.ptr(s), cabi.ptr(y),
                      cabi.ptr(ws) if ws is not None else None, nb,
                      M, N, K, cabi.io_dtype(x2), cabi.fp8_format(w), kind, cabi.current_stream())
        elif s.numel() == 1:
            ops.esimd_gemm_fp8_pert(x2, w, s.reshape(()), y)
        else:
            ops.esimd_gemv_fp8_pern(x2, w, s, y, N, K)
        if bias is not None:
            y += bias
        return y.reshape(*lead, N)
