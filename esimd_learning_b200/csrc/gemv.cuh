// gemv.cuh — launch parameters shared by the FP8 GEMV and its fused
// add+RMSNorm prologue variant.
#pragma once
#include "common.cuh"

namespace cek {

struct GemvParams {
  const void* x;          // [M, K] activations (plain GEMV)
  const uint8_t* w;       // [N, K] fp8
  const void* scale;      // fp16[N] / fp32[N] / fp32[1]
  void* y;                // [M, N]
  int M, N, K;
  int ks;                 // warps per row group (split-K factor)
  int rg_per_cta;         // 16-row groups per CTA
  int mtiles;             // token tiles of 8*NT
  int cpw;                // 64-k chunks per warp
  // fused add+RMSNorm prologue: x = io(residual * inv_rms * gamma)
  const void* residual;   // [M, K] updated residual (written by the stats kernel)
  const void* gamma;      // [K]
  const float* inv_rms;   // [M]
};

// Plans the split-K shape and launches the GEMV (with PDL) on `st`.
int gemv_launch(const GemvParams& base, int x_dtype, int y_dtype, int w_fmt, int scale_kind,
                bool fused, cudaStream_t st);

}  // namespace cek
