// torch_extension_gemm.cc — torch.library registration of the GEMM ops on
// the CUDA dispatch key (fragment of the custom_esimd_kernels_vllm library,
// as in the reference's csrc/xpu/torch_extension_gemm.cc:8-13).
#include <Python.h>

#include "torch_common.h"

using namespace cek_torch;

// Reference: esimd_gemm_fp8_pert (csrc/xpu/esimd_kernel_gemm.sycl:23-64).
// bf16 I/O runs natively (the reference converts through fp16 copies,
// esimd_kernel_gemm.sycl:45-48,61-63).  The reference splits decode (M <= 64,
// GEMV) from prefill (GEMM) at a fixed token count
// (csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:4043-4048); here
// cek_gemm_fp8w_preferred picks by estimated time: the tensor-core GEMV
// family (one weight pass per 16-token tile) for few tokens or few output
// tiles, else the tcgen05 GEMM with the weight converted exactly to 16 bits
// (cek_gemm_fp8w: in shared memory up to 256 tokens, into a workspace first
// above that).

at::Tensor esimd_gemm_fp8_pert(at::Tensor input, at::Tensor weight, at::Tensor weight_scale,
                               at::Tensor output) {
  const char* op = "esimd_gemm_fp8_pert";
  TORCH_CHECK(is_half_or_bf16(input), op, ": input must be fp16 or bf16");
  TORCH_CHECK(is_half_or_bf16(output), op, ": output must be fp16 or bf16");
  TORCH_CHECK(input.scalar_type() == output.scalar_type(), op,
              ": input and output must have the same dtype");
  check_cuda(input, op, "input");
  check_cuda(weight, op, "weight");
  check_cuda(weight_scale, op, "weight_scale");
  check_cuda(output, op, "output");
  TORCH_CHECK(weight.dim() == 2, op, ": weight must be [N, K]");
  TORCH_CHECK(weight_scale.scalar_type() == at::kFloat && weight_scale.numel() == 1, op,
              ": weight_scale must be an fp32 scalar");
  const int64_t N = weight.size(0), K = weight.size(1);
  TORCH_CHECK(input.size(-1) == K, op, ": input must be [M, K]");
  const int64_t M = input.numel() / K;
  TORCH_CHECK(output.numel() == M * N, op, ": output must be [M, N]");
  const int fmt = fp8_format(weight, op);
  c10::cuda::CUDAGuard guard(input.device());
  if (cek_gemm_fp8w_preferred(M, N, K) && input.is_contiguous() && output.is_contiguous() &&
      weight.is_contiguous()) {
    // the 16-bit weight copy is needed only above the in-kernel conversion's rows
    const int64_t ws_bytes = M > CEK_GEMM_FP8W_INKERNEL_MAX_ROWS ? cek_gemm_fp8w_workspace_bytes(N, K) : 0;
    at::Tensor ws = ws_bytes ? at::empty({ws_bytes}, input.options().dtype(at::kByte)) : at::Tensor();
    check_status(cek_gemm_fp8w(input.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(), output.data_ptr(),
                               ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, M, N, K, io_dtype(input), fmt,
                               CEK_SCALE_PERT_F32, stream_of(input)),
                 op);
    return output;
  }
  check_status(cek_gemv_fp8(input.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(),
                            output.data_ptr(), M, N, K, io_dtype(input), io_dtype(output), fmt,
                            CEK_SCALE_PERT_F32, gemv_flags(), stream_of(input)),
               op);
  return output;
}

// New: per-token dynamic e4m3 quantisation: output e4m3 [M, K], scale fp32 [M].
at::Tensor esimd_quant_fp8_per_token(at::Tensor input, at::Tensor output, at::Tensor scale) {
  const char* op = "esimd_quant_fp8_per_token";
  check_cuda(input, op, "input");
  check_cuda(output, op, "output");
  check_cuda(scale, op, "scale");
  TORCH_CHECK(is_half_or_bf16(input), op, ": input must be fp16 or bf16");
  TORCH_CHECK(output.scalar_type() == at::ScalarType::Float8_e4m3fn, op,
              ": output must be float8_e4m3fn");
  TORCH_CHECK(scale.scalar_type() == at::kFloat, op, ": scale must be fp32");
  const int64_t K = input.size(-1);
  const int64_t M = K > 0 ? input.numel() / K : 0;
  TORCH_CHECK(output.numel() == M * K && scale.numel() == M, op, ": output [M, K], scale [M]");
  c10::cuda::CUDAGuard guard(input.device());
  check_status(cek_quant_fp8_per_token(input.data_ptr(), output.data_ptr(),
                                       scale.data_ptr<float>(), M, K, io_dtype(input),
                                       stream_of(input)),
               op);
  return output;
}

// New: prefill FP8 x FP8 GEMM on tcgen05 with per-token x per-channel scales.
// input_q e4m3 [M, K] (esimd_quant_fp8_per_token), input_scale fp32 [M],
// weight e4m3 [N, K], weight_scale fp32 [N], output fp16/bf16 [M, N].
at::Tensor esimd_gemm_fp8_pertoken_pern(at::Tensor input_q, at::Tensor input_scale, at::Tensor weight,
                                        at::Tensor weight_scale, at::Tensor output) {
  const char* op = "esimd_gemm_fp8_pertoken_pern";
  check_cuda(input_q, op, "input_q");
  check_cuda(input_scale, op, "input_scale");
  check_cuda(weight, op, "weight");
  check_cuda(weight_scale, op, "weight_scale");
  check_cuda(output, op, "output");
  TORCH_CHECK(input_q.scalar_type() == at::ScalarType::Float8_e4m3fn &&
                  weight.scalar_type() == at::ScalarType::Float8_e4m3fn,
              op, ": input_q and weight must be float8_e4m3fn");
  TORCH_CHECK(input_scale.scalar_type() == at::kFloat && weight_scale.scalar_type() == at::kFloat, op,
              ": scales must be fp32");
  TORCH_CHECK(is_half_or_bf16(output), op, ": output must be fp16 or bf16");
  TORCH_CHECK(weight.dim() == 2, op, ": weight must be [N, K]");
  const int64_t N = weight.size(0), K = weight.size(1);
  TORCH_CHECK(input_q.size(-1) == K, op, ": input_q must be [M, K]");
  const int64_t M = input_q.numel() / K;
  TORCH_CHECK(input_scale.numel() == M && weight_scale.numel() == N, op,
              ": input_scale [M], weight_scale [N]");
  TORCH_CHECK(output.numel() == M * N, op, ": output must be [M, N]");
  c10::cuda::CUDAGuard guard(input_q.device());
  check_status(cek_gemm_fp8_scaled(input_q.data_ptr(), weight.data_ptr(), input_scale.data_ptr<float>(),
                                   weight_scale.data_ptr<float>(), output.data_ptr(), M, N, K,
                                   io_dtype(output), stream_of(input_q)),
               op);
  return output;
}

TORCH_LIBRARY_FRAGMENT(custom_esimd_kernels_vllm, m) {
  // FP8 GEMM per-tensor scale: input [M, K] fp16, weight [N, K] fp8, output [M, N] fp16
  m.def("esimd_gemm_fp8_pert(Tensor input, Tensor weight, Tensor weight_scale, "
        "Tensor output) -> Tensor");
  m.impl("esimd_gemm_fp8_pert", c10::DispatchKey::CUDA, &esimd_gemm_fp8_pert);

  m.def("esimd_quant_fp8_per_token(Tensor input, Tensor output, Tensor scale) -> Tensor");
  m.impl("esimd_quant_fp8_per_token", c10::DispatchKey::CUDA, &esimd_quant_fp8_per_token);

  m.def("esimd_gemm_fp8_pertoken_pern(Tensor input_q, Tensor input_scale, Tensor weight, "
        "Tensor weight_scale, Tensor output) -> Tensor");
  m.impl("esimd_gemm_fp8_pertoken_pern", c10::DispatchKey::CUDA, &esimd_gemm_fp8_pertoken_pern);
}

PyMODINIT_FUNC PyInit_custom_esimd_kernels_gemm() {
  static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "custom_esimd_kernels_gemm", nullptr,
                                      0, nullptr};
  return PyModule_Create(&module);
}
