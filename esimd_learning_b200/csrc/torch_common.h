// torch_common.h — helpers shared by the two thin torch.library launchers.
// They only validate tensors, pick the enums of include/cek.h and forward raw
// pointers plus the current CUDA stream to libcek_b200.so.
#pragma once
#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <atomic>

#include "cek.h"

namespace cek_torch {

inline void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

inline void check_status(int status, const char* op) {
  TORCH_CHECK(status == CEK_OK, op, ": ", cek_status_string(status), " (status ", status, ")");
}

inline void check_cuda(const at::Tensor& t, const char* op, const char* name) {
  TORCH_CHECK(t.is_cuda(), op, ": ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), op, ": ", name, " must be contiguous");
}

inline int io_dtype(const at::Tensor& t) {
  return t.scalar_type() == at::ScalarType::BFloat16 ? CEK_BF16 : CEK_F16;
}

inline bool is_half_or_bf16(const at::Tensor& t) {
  return t.scalar_type() == at::ScalarType::Half || t.scalar_type() == at::ScalarType::BFloat16;
}

// Reference: fp8 mode from weight.scalar_type(), e5m2 -> 1 else 0
// (csrc/xpu/esimd_kernel.sycl:14-16).  Raw uint8/int8 storage reads as e4m3.
inline int fp8_format(const at::Tensor& w, const char* op) {
  const auto st = w.scalar_type();
  TORCH_CHECK(st == at::ScalarType::Float8_e4m3fn || st == at::ScalarType::Float8_e5m2 ||
                  st == at::ScalarType::Byte || st == at::ScalarType::Char,
              op, ": weight must be float8_e4m3fn, float8_e5m2 or raw 8-bit storage");
  return st == at::ScalarType::Float8_e5m2 ? CEK_E5M2 : CEK_E4M3;
}

// Scale kind from dtype and size: fp16[N] (the reference's per-N scale),
// fp32[N], or an fp32 scalar (per-tensor).
inline int scale_kind(const at::Tensor& s, int64_t N, bool allow_per_tensor, const char* op) {
  if (s.scalar_type() == at::ScalarType::Half) {
    TORCH_CHECK(s.numel() == N, op, ": fp16 weight_scale must have N elements");
    return CEK_SCALE_PERN_F16;
  }
  TORCH_CHECK(s.scalar_type() == at::ScalarType::Float, op,
              ": weight_scale must be fp16[N], fp32[N] or an fp32 scalar");
  if (s.numel() == N && !(allow_per_tensor && N == 1)) return CEK_SCALE_PERN_F32;
  TORCH_CHECK(allow_per_tensor && s.numel() == 1, op, ": weight_scale must have N elements");
  return CEK_SCALE_PERT_F32;
}

// Process-wide switch: let the GEMV ops stream weights before waiting for
// the preceding kernel (CEK_GEMV_EARLY_WEIGHTS).  Off by default; turn it on
// (esimd_set_weight_prefetch) when no kernel writes weights right before a
// GEMV on the same stream, as in a decode step over static weights.
inline std::atomic<bool>& weight_prefetch() {
  static std::atomic<bool> on{false};
  return on;
}
inline unsigned gemv_flags() { return weight_prefetch().load() ? CEK_GEMV_EARLY_WEIGHTS : 0u; }

}  // namespace cek_torch
