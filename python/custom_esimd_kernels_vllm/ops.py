"""Python wrappers of the custom ops (the reference's
python/custom_esimd_kernels_vllm/ops.py:1-67, same names and signatures,
plus the decode-chain ops this build adds).

Every wrapper forwards to `torch.ops.custom_esimd_kernels_vllm.<name>`, which
runs the sm_100a kernels of libcek_b200.so on the current CUDA stream.  Ops
write into caller-provided outputs and return them, as in the reference.
"""
import torch

_ops = torch.ops.custom_esimd_kernels_vllm


def esimd_gemv_fp8_pern(
    input: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
    output: torch.Tensor,
    N: int, K: int,
) -> torch.Tensor:
    """FP8 weight GEMV with per-N scale, FP32 accumulation, scale applied
    after the reduction (reference ops.py:7-18).

    input/output: [M, K]/[M, N] fp16 or bf16 of one dtype (the reference
    takes M = 1; any M works here), weight: [N, K] float8_e4m3fn or
    float8_e5m2, weight_scale: fp16 [N] (as in the reference) or fp32 [N].
    K must be a multiple of 16.
    """
    return _ops.esimd_gemv_fp8_pern(input, weight, weight_scale, output, N, K)


def esimd_gemv_fp8_pern_fused(
    input: torch.Tensor, weights: list, weight_scales: list, outputs: list,
) -> list:
    """Several FP8 GEMVs that share `input`, in one launch (the reference's
    fused multi-GEMV, fp8_GEMV_v2.h:197-316): outputs[i] = input @
    deq(weights[i])^T * weight_scales[i], for 1 to 4 matrices with one FP8
    format and one scale kind.  Returns outputs."""
    _ops.esimd_gemv_fp8_pern_fused(input, weights, weight_scales, outputs)
    return outputs


def esimd_gemv_fp8_pert(
    input: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
    output: torch.Tensor,
) -> torch.Tensor:
    """FP8 weight GEMV with per-tensor scale (fp32 scalar read on the device),
    N and K from weight.shape (reference ops.py:22-32)."""
    return _ops.esimd_gemv_fp8_pert(input, weight, weight_scale, output)


def esimd_fused_add_rms_norm_batched(
    hidden_states: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
) -> torch.Tensor:
    """Batched residual add + RMSNorm, Gemma style (reference ops.py:34-46).

    residual[i] = hidden_states[i] + residual[i]  (in place)
    hidden_states[i] = rmsnorm(residual[i]) * weight  (in place, returned)
    weight must be pre-adjusted (w + 1.0).  K % 8 == 0, K <= 16384.
    """
    return _ops.esimd_fused_add_rms_norm_batched(hidden_states, residual, weight, eps)


def esimd_gemm_fp8_pert(
    input: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
    output: torch.Tensor,
) -> torch.Tensor:
    """FP8 GEMM with per-tensor scale for any M (reference ops.py:49-67).

    input/output: [M, K]/[M, N] fp16 or bf16 of one dtype, weight: [N, K]
    fp8, weight_scale: fp32 scalar.  bf16 runs natively (no fp16 copies).
    """
    return _ops.esimd_gemm_fp8_pert(input, weight, weight_scale, output)


def esimd_fused_add_rms_norm_batched_fp8(
    hidden_states: torch.Tensor,
    residual: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    qweight: torch.Tensor,
    qweight_scale: torch.Tensor,
    output: torch.Tensor,
) -> torch.Tensor:
    """Residual add + RMSNorm feeding an FP8 GEMV, in two launches chained by
    programmatic dependent launch; the normalised activation never goes to HBM.

    residual = hidden_states + residual (in place); hidden_states is only read.
    output[M, N] = rmsnorm(residual) * weight @ deq(qweight)^T * qweight_scale.
    weight: pre-shifted (w + 1.0) [K]; qweight [N, K] fp8; qweight_scale fp16/fp32
    [N] or fp32 scalar.  M <= 16.
    """
    return _ops.esimd_fused_add_rms_norm_batched_fp8(
        hidden_states, residual, weight, eps, qweight, qweight_scale, output)


def esimd_gelu_and_mul(input: torch.Tensor, output: torch.Tensor) -> torch.Tensor:
    """output[..., j] = gelu_tanh(input[..., j]) * input[..., d + j], d = input.shape[-1] // 2."""
    return _ops.esimd_gelu_and_mul(input, output)


def esimd_gemv_fp8_gelu_mul(input: torch.Tensor, weight: torch.Tensor, weight_scale: torch.Tensor,
                            output: torch.Tensor) -> torch.Tensor:
    """output [M, N] = gelu_tanh(g) * u, [g | u] = GEMV(input, weight [2N, K] fp8 with gate rows
    then up rows, weight_scale [2N] or scalar), each half rounded to the io dtype first: the
    gate_up projection with GeLU-and-mul fused into its epilogue."""
    return _ops.esimd_gemv_fp8_gelu_mul(input, weight, weight_scale, output)


def esimd_fused_add_rms_norm_gelu_mul_fp8(hidden_states: torch.Tensor, residual: torch.Tensor,
                                          weight: torch.Tensor, eps: float, qweight: torch.Tensor,
                                          qweight_scale: torch.Tensor, output: torch.Tensor) -> torch.Tensor:
    """esimd_fused_add_rms_norm_batched_fp8 with the gated projection of esimd_gemv_fp8_gelu_mul:
    residual += hidden; output [M, N] = gelu(g) * u of GEMV(RMSNorm(residual) * weight, qweight [2N, K])."""
    return _ops.esimd_fused_add_rms_norm_gelu_mul_fp8(hidden_states, residual, weight, eps, qweight,
                                                      qweight_scale, output)


def esimd_qkv_norm_rope(
    qkv: torch.Tensor, positions: torch.Tensor, q_weight: torch.Tensor,
    k_weight: torch.Tensor, cos_sin_cache: torch.Tensor,
    num_q_heads: int, num_kv_heads: int, head_dim: int, eps: float,
    is_neox: bool = True,
) -> torch.Tensor:
    """In place on qkv [M, (Hq + 2 Hkv) * D]: per-head RMSNorm of the q and k
    heads (weights q_weight / k_weight [D]), then rotary embedding at
    `positions` (int64 [M]) from cos_sin_cache fp32 [max_pos, D] (cos | sin
    halves).  v heads are untouched.  Returns qkv."""
    return _ops.esimd_qkv_norm_rope(qkv, positions, q_weight, k_weight, cos_sin_cache,
                                    num_q_heads, num_kv_heads, head_dim, eps, is_neox)


def esimd_quant_fp8_per_token(
    input: torch.Tensor, output: torch.Tensor, scale: torch.Tensor,
) -> torch.Tensor:
    """Dynamic per-token e4m3 quantisation: scale[m] = max(amax_m, 1e-12) / 448,
    output = e4m3(clamp(input / scale[m], -448, 448)).  Returns output."""
    return _ops.esimd_quant_fp8_per_token(input, output, scale)


def esimd_set_weight_prefetch(enable: bool) -> bool:
    """Let the FP8 GEMV ops start streaming weights before the preceding
    kernel on the stream has finished (programmatic dependent launch), which
    hides launch and DRAM latency between back-to-back decode kernels.  Only
    valid while no kernel writes a GEMV's weights immediately before that
    GEMV on the same stream (true for static model weights).  Process-wide;
    returns the previous setting."""
    return _ops.esimd_set_weight_prefetch(enable)


def esimd_gemm_fp8_pertoken_pern(
    input_q: torch.Tensor, input_scale: torch.Tensor, weight: torch.Tensor,
    weight_scale: torch.Tensor, output: torch.Tensor,
) -> torch.Tensor:
    """Prefill FP8 GEMM on the Blackwell tensor cores (tcgen05):
    output = (deq(input_q) @ deq(weight)^T) * input_scale[:, None] * weight_scale[None, :].

    input_q e4m3 [M, K] with input_scale fp32 [M] (from esimd_quant_fp8_per_token),
    weight e4m3 [N, K] with weight_scale fp32 [N], output fp16/bf16 [M, N].
    K % 128 == 0, N % 16 == 0.  Returns output."""
    return _ops.esimd_gemm_fp8_pertoken_pern(input_q, input_scale, weight, weight_scale, output)
