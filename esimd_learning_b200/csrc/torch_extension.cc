// torch_extension.cc — torch.library registration of the GEMV / add+RMSNorm
// ops on the CUDA dispatch key, and the decode-chain helper ops.
//
// The three reference schemas are kept byte for byte
// (csrc/xpu/torch_extension.cc:9-18); only the dispatch key changes from
// kXPU to kCUDA.  Each op validates its tensors (the reference's dtype
// TORCH_CHECKs, esimd_kernel.sycl:26-37 and :62-73, plus device, contiguity
// and size checks), forwards raw pointers and the current CUDA stream to the
// C ABI of libcek_b200.so, and returns the tensor it wrote, as the reference
// does (esimd_kernel.sycl:52, :88, :108).
#include <Python.h>

#include "torch_common.h"

using namespace cek_torch;

namespace {

void check_gemv_io(const at::Tensor& input, const at::Tensor& output, const char* op) {
  TORCH_CHECK(is_half_or_bf16(input), op, ": input must be fp16 or bf16");
  TORCH_CHECK(is_half_or_bf16(output), op, ": output must be fp16 or bf16");
  TORCH_CHECK(input.scalar_type() == output.scalar_type(), op,
              ": input and output must have the same dtype");
}

at::Tensor run_gemv(const char* op, at::Tensor& input, const at::Tensor& weight,
                    const at::Tensor& scale, at::Tensor& output, int64_t N, int64_t K,
                    bool allow_per_tensor) {
  check_gemv_io(input, output, op);
  check_cuda(input, op, "input");
  check_cuda(weight, op, "weight");
  check_cuda(scale, op, "weight_scale");
  check_cuda(output, op, "output");
  TORCH_CHECK(N > 0 && K > 0, op, ": N and K must be positive");
  TORCH_CHECK(weight.numel() == N * K, op, ": weight must hold N*K elements");
  TORCH_CHECK(input.numel() % K == 0, op, ": input numel must be a multiple of K");
  const int64_t M = input.numel() / K;
  TORCH_CHECK(output.numel() == M * N, op, ": output must hold M*N elements");
  const int fmt = fp8_format(weight, op);
  const int sk = scale_kind(scale, N, allow_per_tensor, op);
  c10::cuda::CUDAGuard guard(input.device());
  check_status(cek_gemv_fp8(input.data_ptr(), weight.data_ptr(), scale.data_ptr(),
                            output.data_ptr(), M, N, K, io_dtype(input), io_dtype(output), fmt,
                            sk, gemv_flags(), stream_of(input)),
               op);
  return output;
}

}  // namespace

// Reference: esimd_gemv_fp8_pern (csrc/xpu/esimd_kernel.sycl:22-53).  Also
// accepts input [M, K] (M = input.numel() / K) and an fp32 [N] scale.
at::Tensor esimd_gemv_fp8_pern(at::Tensor input, at::Tensor weight, at::Tensor weight_scale,
                               at::Tensor output, int64_t N, int64_t K) {
  return run_gemv("esimd_gemv_fp8_pern", input, weight, weight_scale, output, N, K, false);
}

// New op, the reference's fused multi-GEMV (fp8_GEMV_v2.h:197-316, compiled
// there but not registered): outputs[i] = GEMV(input, weights[i], scales[i])
// for up to 4 matrices sharing input, in one launch.
void esimd_gemv_fp8_pern_fused(at::Tensor input, std::vector<at::Tensor> weights,
                               std::vector<at::Tensor> weight_scales, std::vector<at::Tensor> outputs) {
  const char* op = "esimd_gemv_fp8_pern_fused";
  const size_t n = weights.size();
  TORCH_CHECK(n >= 1 && n <= 4 && weight_scales.size() == n && outputs.size() == n, op,
              ": 1 to 4 weights, with one scale and one output each");
  check_cuda(input, op, "input");
  TORCH_CHECK(is_half_or_bf16(input), op, ": input must be fp16 or bf16");
  const int64_t K = weights[0].size(-1);
  TORCH_CHECK(K > 0 && input.numel() % K == 0, op, ": input numel must be a multiple of K");
  const int64_t M = input.numel() / K;
  const void* wp[4];
  const void* sp[4];
  void* yp[4];
  int64_t ns[4];
  int fmt = -1, sk = -1;
  for (size_t i = 0; i < n; ++i) {
    check_cuda(weights[i], op, "weight");
    check_cuda(weight_scales[i], op, "weight_scale");
    check_cuda(outputs[i], op, "output");
    TORCH_CHECK(weights[i].dim() == 2 && weights[i].size(1) == K, op, ": weights must be [N_i, K]");
    TORCH_CHECK(outputs[i].scalar_type() == input.scalar_type(), op, ": outputs must match the input dtype");
    ns[i] = weights[i].size(0);
    TORCH_CHECK(outputs[i].numel() == M * ns[i], op, ": output i must be [M, N_i]");
    const int f = fp8_format(weights[i], op), k = scale_kind(weight_scales[i], ns[i], true, op);
    TORCH_CHECK((fmt < 0 || f == fmt) && (sk < 0 || k == sk), op,
                ": all weights must share one FP8 format and one scale kind");
    fmt = f;
    sk = k;
    wp[i] = weights[i].data_ptr();
    sp[i] = weight_scales[i].data_ptr();
    yp[i] = outputs[i].data_ptr();
  }
  c10::cuda::CUDAGuard guard(input.device());
  check_status(cek_gemv_fp8_multi(input.data_ptr(), wp, sp, yp, ns, (int)n, M, K, io_dtype(input),
                                  io_dtype(input), fmt, sk, gemv_flags(), stream_of(input)),
               op);
}

// Reference: esimd_gemv_fp8_pert (csrc/xpu/esimd_kernel.sycl:57-89); N, K from weight.
at::Tensor esimd_gemv_fp8_pert(at::Tensor input, at::Tensor weight, at::Tensor weight_scale,
                               at::Tensor output) {
  const char* op = "esimd_gemv_fp8_pert";
  TORCH_CHECK(weight.dim() == 2, op, ": weight must be [N, K]");
  TORCH_CHECK(weight_scale.scalar_type() == at::ScalarType::Float && weight_scale.numel() == 1, op,
              ": weight_scale must be an fp32 scalar");
  return run_gemv(op, input, weight, weight_scale, output, weight.size(0), weight.size(1), true);
}

// Reference: esimd_fused_add_rms_norm_batched (csrc/xpu/esimd_kernel.sycl:90-108).
at::Tensor esimd_fused_add_rms_norm_batched(at::Tensor hidden_states, at::Tensor residual,
                                            at::Tensor weight, double eps) {
  const char* op = "esimd_fused_add_rms_norm_batched";
  check_cuda(hidden_states, op, "hidden_states");
  check_cuda(residual, op, "residual");
  check_cuda(weight, op, "weight");
  TORCH_CHECK(is_half_or_bf16(hidden_states), op, ": hidden_states must be fp16 or bf16");
  TORCH_CHECK(residual.scalar_type() == hidden_states.scalar_type() &&
                  weight.scalar_type() == hidden_states.scalar_type(),
              op, ": hidden_states, residual and weight must share a dtype");
  const int64_t K = hidden_states.size(-1);
  TORCH_CHECK(residual.numel() == hidden_states.numel(), op, ": residual shape mismatch");
  TORCH_CHECK(weight.numel() == K, op, ": weight must have K elements");
  const int64_t rows = K > 0 ? hidden_states.numel() / K : 0;
  c10::cuda::CUDAGuard guard(hidden_states.device());
  check_status(cek_fused_add_rmsnorm(hidden_states.data_ptr(), residual.data_ptr(),
                                     weight.data_ptr(), rows, K, (float)eps,
                                     io_dtype(hidden_states), stream_of(hidden_states)),
               op);
  return hidden_states;
}

// New: residual add + RMSNorm fused into the prologue of an FP8 GEMV.
// residual is updated in place, hidden_states is only read; returns output.
at::Tensor esimd_fused_add_rms_norm_batched_fp8(at::Tensor hidden_states, at::Tensor residual,
                                                at::Tensor weight, double eps, at::Tensor qweight,
                                                at::Tensor qweight_scale, at::Tensor output) {
  const char* op = "esimd_fused_add_rms_norm_batched_fp8";
  check_cuda(hidden_states, op, "hidden_states");
  check_cuda(residual, op, "residual");
  check_cuda(weight, op, "weight");
  check_cuda(qweight, op, "qweight");
  check_cuda(qweight_scale, op, "qweight_scale");
  check_cuda(output, op, "output");
  TORCH_CHECK(is_half_or_bf16(hidden_states), op, ": hidden_states must be fp16 or bf16");
  TORCH_CHECK(residual.scalar_type() == hidden_states.scalar_type() &&
                  weight.scalar_type() == hidden_states.scalar_type() &&
                  output.scalar_type() == hidden_states.scalar_type(),
              op, ": hidden_states, residual, weight and output must share a dtype");
  TORCH_CHECK(qweight.dim() == 2, op, ": qweight must be [N, K]");
  const int64_t N = qweight.size(0), K = qweight.size(1);
  TORCH_CHECK(hidden_states.size(-1) == K && residual.numel() == hidden_states.numel(), op,
              ": hidden_states/residual must be [M, K]");
  TORCH_CHECK(weight.numel() == K, op, ": weight must have K elements");
  const int64_t M = hidden_states.numel() / K;
  TORCH_CHECK(output.numel() == M * N, op, ": output must hold M*N elements");
  const int fmt = fp8_format(qweight, op);
  const int sk = scale_kind(qweight_scale, N, true, op);
  c10::cuda::CUDAGuard guard(hidden_states.device());
  TORCH_CHECK(M <= 16, op, ": at most 16 rows");
  // normalised rows (M x K): a small caching-allocator block (graph-safe)
  const int64_t ws_bytes = cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K);
  at::Tensor ws = at::empty({ws_bytes}, hidden_states.options().dtype(at::kByte));
  check_status(cek_fused_add_rmsnorm_gemv_fp8(
                   hidden_states.data_ptr(), residual.data_ptr(), weight.data_ptr(), (float)eps,
                   qweight.data_ptr(), qweight_scale.data_ptr(), output.data_ptr(), ws.data_ptr(),
                   ws_bytes, M, N, K, io_dtype(hidden_states), fmt, sk, 0u,
                   stream_of(hidden_states)),
               op);
  return output;
}

// New: out = gelu_tanh(input[:, :d]) * input[:, d:].
at::Tensor esimd_gelu_and_mul(at::Tensor input, at::Tensor output) {
  const char* op = "esimd_gelu_and_mul";
  check_cuda(input, op, "input");
  check_cuda(output, op, "output");
  TORCH_CHECK(is_half_or_bf16(input) && output.scalar_type() == input.scalar_type(), op,
              ": input and output must be fp16 or bf16 of one dtype");
  const int64_t two_d = input.size(-1);
  TORCH_CHECK(two_d % 2 == 0, op, ": last dim of input must be even");
  const int64_t d = two_d / 2;
  const int64_t M = d > 0 ? input.numel() / two_d : 0;
  TORCH_CHECK(output.numel() == M * d, op, ": output must be [..., d]");
  c10::cuda::CUDAGuard guard(input.device());
  check_status(cek_gelu_and_mul(input.data_ptr(), output.data_ptr(), M, d, io_dtype(input),
                                stream_of(input)),
               op);
  return output;
}

// New: output [M, N] = gelu_tanh(g) * u with [g | u] = GEMV(input, weight
// [2N, K]) rounded to the io dtype: the decode MLP's gate_up projection with
// GeLU-and-mul fused into its epilogue (cek_gemv_fp8 with
// CEK_GEMV_GELU_MUL_OUTPUT).  Shapes the fused kernel does not take run as
// the GEMV into a [M, 2N] temporary followed by esimd_gelu_and_mul, which is
// the same arithmetic.
at::Tensor esimd_gemv_fp8_gelu_mul(at::Tensor input, at::Tensor weight, at::Tensor weight_scale,
                                   at::Tensor output) {
  const char* op = "esimd_gemv_fp8_gelu_mul";
  check_cuda(input, op, "input");
  check_cuda(weight, op, "weight");
  check_cuda(weight_scale, op, "weight_scale");
  check_cuda(output, op, "output");
  check_gemv_io(input, output, op);
  TORCH_CHECK(weight.dim() == 2 && weight.size(0) % 2 == 0, op, ": weight must be [2N, K]");
  const int64_t N = weight.size(0) / 2, K = weight.size(1);
  TORCH_CHECK(K > 0 && input.size(-1) == K, op, ": input must be [M, K]");
  const int64_t M = input.numel() / K;
  TORCH_CHECK(output.numel() == M * N, op, ": output must be [M, N]");
  const int fmt = fp8_format(weight, op);
  const int sk = scale_kind(weight_scale, 2 * N, true, op);
  c10::cuda::CUDAGuard guard(input.device());
  const int rc = cek_gemv_fp8(input.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(), output.data_ptr(), M, N,
                              K, io_dtype(input), io_dtype(output), fmt, sk, gemv_flags() | CEK_GEMV_GELU_MUL_OUTPUT,
                              stream_of(input));
  if (rc != CEK_ERR_UNSUPPORTED) {
    check_status(rc, op);
    return output;
  }
  at::Tensor gu = at::empty({M, 2 * N}, output.options());
  check_status(cek_gemv_fp8(input.data_ptr(), weight.data_ptr(), weight_scale.data_ptr(), gu.data_ptr(), M, 2 * N,
                            K, io_dtype(input), io_dtype(gu), fmt, sk, gemv_flags(), stream_of(input)),
               op);
  check_status(cek_gelu_and_mul(gu.data_ptr(), output.data_ptr(), M, N, io_dtype(gu), stream_of(input)), op);
  return output;
}

// New: esimd_fused_add_rms_norm_batched_fp8 whose projection is the gated
// gate_up one above: residual += hidden; hidden = RMSNorm(residual) * weight;
// output [M, N] = gelu_tanh(g) * u, [g | u] = GEMV(hidden, qweight [2N, K]).
at::Tensor esimd_fused_add_rms_norm_gelu_mul_fp8(at::Tensor hidden_states, at::Tensor residual, at::Tensor weight,
                                                 double eps, at::Tensor qweight, at::Tensor qweight_scale,
                                                 at::Tensor output) {
  const char* op = "esimd_fused_add_rms_norm_gelu_mul_fp8";
  check_cuda(hidden_states, op, "hidden_states");
  check_cuda(residual, op, "residual");
  check_cuda(weight, op, "weight");
  check_cuda(qweight, op, "qweight");
  check_cuda(qweight_scale, op, "qweight_scale");
  check_cuda(output, op, "output");
  TORCH_CHECK(is_half_or_bf16(hidden_states), op, ": hidden_states must be fp16 or bf16");
  TORCH_CHECK(residual.scalar_type() == hidden_states.scalar_type() &&
                  weight.scalar_type() == hidden_states.scalar_type() &&
                  output.scalar_type() == hidden_states.scalar_type(),
              op, ": hidden_states, residual, weight and output must share a dtype");
  TORCH_CHECK(qweight.dim() == 2 && qweight.size(0) % 2 == 0, op, ": qweight must be [2N, K]");
  const int64_t N = qweight.size(0) / 2, K = qweight.size(1);
  TORCH_CHECK(hidden_states.size(-1) == K && residual.numel() == hidden_states.numel(), op,
              ": hidden_states/residual must be [M, K]");
  TORCH_CHECK(weight.numel() == K, op, ": weight must have K elements");
  const int64_t M = hidden_states.numel() / K;
  TORCH_CHECK(M <= 16, op, ": at most 16 rows");
  TORCH_CHECK(output.numel() == M * N, op, ": output must hold M*N elements");
  const int fmt = fp8_format(qweight, op);
  const int sk = scale_kind(qweight_scale, 2 * N, true, op);
  c10::cuda::CUDAGuard guard(hidden_states.device());
  const int64_t ws_bytes = cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K);
  at::Tensor ws = at::empty({ws_bytes}, hidden_states.options().dtype(at::kByte));
  const bool fused = M <= 16 && K % 64 == 0;  // what the gated bulk GEMV takes
  at::Tensor gu = fused ? output : at::empty({M, 2 * N}, output.options());
  check_status(cek_fused_add_rmsnorm_gemv_fp8(hidden_states.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                              (float)eps, qweight.data_ptr(), qweight_scale.data_ptr(), gu.data_ptr(),
                                              ws.data_ptr(), ws_bytes, M, fused ? N : 2 * N, K,
                                              io_dtype(hidden_states), fmt, sk,
                                              fused ? CEK_GEMV_GELU_MUL_OUTPUT : 0u, stream_of(hidden_states)),
               op);
  if (!fused)
    check_status(cek_gelu_and_mul(gu.data_ptr(), output.data_ptr(), M, N, io_dtype(gu), stream_of(hidden_states)),
                 op);
  return output;
}

// New: per-head RMSNorm on q and k heads, then rotary embedding, in place.
at::Tensor esimd_qkv_norm_rope(at::Tensor qkv, at::Tensor positions, at::Tensor q_weight,
                               at::Tensor k_weight, at::Tensor cos_sin_cache, int64_t num_q_heads,
                               int64_t num_kv_heads, int64_t head_dim, double eps, bool is_neox) {
  const char* op = "esimd_qkv_norm_rope";
  check_cuda(qkv, op, "qkv");
  check_cuda(positions, op, "positions");
  check_cuda(q_weight, op, "q_weight");
  check_cuda(k_weight, op, "k_weight");
  check_cuda(cos_sin_cache, op, "cos_sin_cache");
  TORCH_CHECK(is_half_or_bf16(qkv), op, ": qkv must be fp16 or bf16");
  TORCH_CHECK(q_weight.scalar_type() == qkv.scalar_type() &&
                  k_weight.scalar_type() == qkv.scalar_type(),
              op, ": norm weights must match the qkv dtype");
  TORCH_CHECK(positions.scalar_type() == at::kLong, op, ": positions must be int64");
  TORCH_CHECK(cos_sin_cache.scalar_type() == at::kFloat && cos_sin_cache.dim() == 2 &&
                  cos_sin_cache.size(1) == head_dim,
              op, ": cos_sin_cache must be fp32 [max_position, head_dim]");
  TORCH_CHECK(q_weight.numel() == head_dim && k_weight.numel() == head_dim, op,
              ": norm weights must have head_dim elements");
  const int64_t width = (num_q_heads + 2 * num_kv_heads) * head_dim;
  TORCH_CHECK(width > 0 && qkv.size(-1) == width, op, ": qkv last dim must be (Hq + 2 Hkv) * D");
  const int64_t M = qkv.numel() / width;
  TORCH_CHECK(positions.numel() == M, op, ": positions must have one entry per token");
  c10::cuda::CUDAGuard guard(qkv.device());
  check_status(cek_qkv_norm_rope(qkv.data_ptr(), positions.data_ptr<int64_t>(),
                                 q_weight.data_ptr(), k_weight.data_ptr(),
                                 cos_sin_cache.data_ptr<float>(), M, num_q_heads, num_kv_heads,
                                 head_dim, cos_sin_cache.size(0), (float)eps, is_neox ? 1 : 0,
                                 io_dtype(qkv), stream_of(qkv)),
               op);
  return qkv;
}

// New: process-wide switch for CEK_GEMV_EARLY_WEIGHTS; returns the old value.
bool esimd_set_weight_prefetch(bool enable) { return weight_prefetch().exchange(enable); }

TORCH_LIBRARY(custom_esimd_kernels_vllm, m) {
  m.def("esimd_gemv_fp8_pern(Tensor input, Tensor weight, Tensor weight_scale, "
        "Tensor output, int N, int K) -> Tensor");
  m.impl("esimd_gemv_fp8_pern", c10::DispatchKey::CUDA, &esimd_gemv_fp8_pern);

  m.def("esimd_gemv_fp8_pert(Tensor input, Tensor weight, Tensor weight_scale, "
        "Tensor output) -> Tensor");
  m.impl("esimd_gemv_fp8_pert", c10::DispatchKey::CUDA, &esimd_gemv_fp8_pert);
  m.def("esimd_fused_add_rms_norm_batched(Tensor hidden_states, Tensor residual, "
        "Tensor weight, float eps) -> Tensor");
  m.impl("esimd_fused_add_rms_norm_batched", c10::DispatchKey::CUDA, &esimd_fused_add_rms_norm_batched);

  m.def("esimd_gemv_fp8_pern_fused(Tensor input, Tensor[] weights, Tensor[] weight_scales, "
        "Tensor(a!)[] outputs) -> ()");
  m.impl("esimd_gemv_fp8_pern_fused", c10::DispatchKey::CUDA, &esimd_gemv_fp8_pern_fused);

  m.def("esimd_fused_add_rms_norm_batched_fp8(Tensor hidden_states, Tensor residual, "
        "Tensor weight, float eps, Tensor qweight, Tensor qweight_scale, Tensor output) -> Tensor");
  m.impl("esimd_fused_add_rms_norm_batched_fp8", c10::DispatchKey::CUDA,
         &esimd_fused_add_rms_norm_batched_fp8);
  m.def("esimd_gelu_and_mul(Tensor input, Tensor output) -> Tensor");
  m.impl("esimd_gelu_and_mul", c10::DispatchKey::CUDA, &esimd_gelu_and_mul);
  m.def("esimd_gemv_fp8_gelu_mul(Tensor input, Tensor weight, Tensor weight_scale, Tensor output) -> Tensor");
  m.impl("esimd_gemv_fp8_gelu_mul", c10::DispatchKey::CUDA, &esimd_gemv_fp8_gelu_mul);
  m.def("esimd_fused_add_rms_norm_gelu_mul_fp8(Tensor hidden_states, Tensor residual, Tensor weight, float eps, "
        "Tensor qweight, Tensor qweight_scale, Tensor output) -> Tensor");
  m.impl("esimd_fused_add_rms_norm_gelu_mul_fp8", c10::DispatchKey::CUDA, &esimd_fused_add_rms_norm_gelu_mul_fp8);
  m.def("esimd_qkv_norm_rope(Tensor qkv, Tensor positions, Tensor q_weight, Tensor k_weight, "
        "Tensor cos_sin_cache, int num_q_heads, int num_kv_heads, int head_dim, float eps, "
        "bool is_neox) -> Tensor");
  m.impl("esimd_qkv_norm_rope", c10::DispatchKey::CUDA, &esimd_qkv_norm_rope);
  m.def("esimd_set_weight_prefetch(bool enable) -> bool", &esimd_set_weight_prefetch);
}

PyMODINIT_FUNC PyInit_custom_esimd_kernels() {
  static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "custom_esimd_kernels", nullptr, 0,
                                      nullptr};
  return PyModule_Create(&module);
}
