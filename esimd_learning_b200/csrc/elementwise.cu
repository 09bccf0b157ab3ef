// elementwise.cu — the decode-step helpers around the FP8 GEMVs:
//   * GeLU(tanh)-and-mul            (cek_gelu_and_mul)
//   * q/k per-head RMSNorm + RoPE   (cek_qkv_norm_rope)
//   * per-token dynamic e4m3 quant  (cek_quant_fp8_per_token)
// None has a counterpart kernel in the reference (it ships only the GEMV, the
// GEMM and add+RMSNorm); they complete the decode chain whose GEMVs it does
// ship.  All are HBM-bound: 16-byte vector loads and stores, fp32 math,
// one rounding to the I/O type per stored value.
#include "common.cuh"
#include <cuda_fp8.h>

namespace cek {

// ---- GeLU(tanh)-and-mul -----------------------------------------------------
// out[m, j] = io( gelu_tanh(f32 x[m, j]) * f32 x[m, d + j] ),
// gelu_tanh(g) = 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))).
template <typename T>
__global__ void __launch_bounds__(256)
gelu_and_mul_kernel(const T* __restrict__ x, T* __restrict__ out, int d) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;  // 8-element group index
  if (v * 8 >= d) return;
  const T* row = x + (size_t)m * 2 * d;
  if (d % 8 == 0) {
    const uint4 gv = *reinterpret_cast<const uint4*>(row + v * 8);
    const uint4 uv = *reinterpret_cast<const uint4*>(row + d + v * 8);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t ow[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) ow[q] = gelu_mul2<T>(gw[q], uw[q]);
    *reinterpret_cast<uint4*>(out + (size_t)m * d + v * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  } else {
    // rows not 16-byte aligned: element by element, same arithmetic
    for (int j = v * 8; j < min(d, v * 8 + 8); ++j) out[(size_t)m * d + j] = gelu_mul1<T>(row[j], row[d + j]);
  }
}

// ---- q/k per-head RMSNorm + rotary embedding -----------------------------------
// One warp per (token, head) over the q and k heads; v heads are not touched.
// E = D / 64 elements per half-head per lane.
//   neox (rotate-half): lane holds x[l*E .. l*E+E) and x[D/2 + l*E ..); pair
//     (i, i + D/2) rotates by angle index i.
//   interleaved: lane holds x[2lE .. 2lE + 2E); pair (2i, 2i+1) rotates by i.
// xn = io(x * rsqrt(mean(x^2) + eps) * w); out = io(rotate(f32 xn)).
template <typename T, int E, bool NEOX>
__global__ void __launch_bounds__(256)
qkv_norm_rope_kernel(T* qkv, const int64_t* __restrict__ pos, const T* __restrict__ qw,
                     const T* __restrict__ kw, const float* __restrict__ cos_sin, int M, int hq,
                     int hkv, int max_pos, float eps) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int D = 64 * E;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = hq + hkv;
  if (gw >= M * heads) return;
  const int m = gw / heads, h = gw % heads;
  T* head = qkv + (size_t)m * (hq + 2 * hkv) * D + (size_t)h * D;
  const T* w = h < hq ? qw : kw;
  int64_t p = pos[m];
  p = p < 0 ? 0 : (p >= max_pos ? max_pos - 1 : p);
  const float* cs = cos_sin + (size_t)p * D;

  float x[2 * E];
  int idx[2 * E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    idx[e] = NEOX ? lane * E + e : lane * 2 * E + e;
    idx[E + e] = NEOX ? D / 2 + lane * E + e : lane * 2 * E + E + e;
  }
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) x[e] = to_f32<T>(head[idx[e]]);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) ss += x[e] * x[e];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) x[e] = to_f32<T>(from_f32<T>(x[e] * inv * to_f32<T>(w[idx[e]])));
  float o[2 * E];
  if constexpr (NEOX) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = lane * E + e;
      const float c = cs[i], s = cs[D / 2 + i];
      o[e] = x[e] * c - x[E + e] * s;
      o[E + e] = x[E + e] * c + x[e] * s;
    }
  } else {
#pragma unroll
    for (int q = 0; q < E; ++q) {
      const int i = lane * E + q;  // pair index
      const float c = cs[i], s = cs[D / 2 + i];
      const float x0 = x[2 * q], x1 = x[2 * q + 1];
      o[2 * q] = x0 * c - x1 * s;
      o[2 * q + 1] = x1 * c + x0 * s;
    }
  }
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) head[idx[e]] = from_f32<T>(o[e]);
}

// ---- per-token dynamic e4m3 quantisation -------------------------------------
// s = max(amax, 1e-12) / 448 with IEEE division; q = e4m3_rn_sat(a / s).
// One CTA per row, 256 threads; the row stays in registers between the amax
// reduction and the quantisation (VPT 16-byte vectors per thread, K <= 16384),
// so it is read from HBM once.
template <typename T, int VPT>
__global__ void __launch_bounds__(256)
quant_fp8_per_token_kernel(const T* __restrict__ a, uint8_t* __restrict__ q, float* __restrict__ sc,
                           int K) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const T* row = a + (size_t)m * K;
  const int nvec = K >> 3;
  uint4 v[VPT];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * 256;
    v[i] = idx < nvec ? *reinterpret_cast<const uint4*>(row + idx * 8) : make_uint4(0, 0, 0, 0);
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack2<T>(w[j]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? sh[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) sh[0] = t;
  }
  __syncthreads();
  const float s = __fdiv_rn(fmaxf(sh[0], 1e-12f), 448.f);
  if (threadIdx.x == 0) sc[m] = s;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = threadIdx.x + i * 256;
    if (idx >= nvec) continue;
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack2<T>(w[j]);
      float2 r;
      r.x = fminf(fmaxf(__fdiv_rn(f.x, s), -448.f), 448.f);
      r.y = fminf(fmaxf(__fdiv_rn(f.y, s), -448.f), 448.f);
      const __nv_fp8x2_storage_t p2 = __nv_cvt_float2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
      packed[j >> 1] |= (uint32_t)p2 << (16 * (j & 1));
    }
    *reinterpret_cast<uint2*>(q + (size_t)m * K + idx * 8) = make_uint2(packed[0], packed[1]);
  }
}

}  // namespace cek

extern "C" int cek_gelu_and_mul(const void* x, void* out, int64_t M, int64_t d, int dtype,
                                void* stream) {
  if (M < 0 || d < 0 || M > 65535) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (M == 0 || d == 0) return CEK_OK;
  if (!x || !out) return CEK_ERR_INVALID_ARG;
  if (d % 8 == 0 && (!cek_host::aligned16(x) || !cek_host::aligned16(out))) return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)(((d + 7) / 8 + 255) / 256), (unsigned)M), block(256);
  if (dtype == CEK_F16)
    return cek_host::launch_pdl(cek::gelu_and_mul_kernel<__half>, grid, block, 0, st, x, out, (int)d);
  return cek_host::launch_pdl(cek::gelu_and_mul_kernel<__nv_bfloat16>, grid, block, 0, st, x, out, (int)d);
}

extern "C" int cek_qkv_norm_rope(void* qkv, const int64_t* positions, const void* q_weight,
                                 const void* k_weight, const float* cos_sin_cache, int64_t M,
                                 int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                                 int64_t max_position, float eps, int is_neox, int dtype,
                                 void* stream) {
  if (M < 0 || num_q_heads < 0 || num_kv_heads < 0 || max_position <= 0) return CEK_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  const int64_t warps = M * (num_q_heads + num_kv_heads);
  if (warps == 0) return CEK_OK;
  if (!qkv || !positions || !q_weight || !k_weight || !cos_sin_cache) return CEK_ERR_INVALID_ARG;
  if (warps * 32 > (int64_t)INT32_MAX) return CEK_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)((warps * 32 + 255) / 256)), block(256);
  const int m = (int)M, hq = (int)num_q_heads, hkv = (int)num_kv_heads, mp = (int)max_position;
  int s = CEK_OK;
#define CEK_ROPE(T, E, NX)                                                                       \
  s = cek_host::launch_pdl(cek::qkv_norm_rope_kernel<T, E, NX>, grid, block, 0, st, qkv, positions,  \
                           q_weight, k_weight, cos_sin_cache, m, hq, hkv, mp, eps)
#define CEK_ROPE_E(T, NX)                                       \
  if (head_dim == 64) CEK_ROPE(T, 1, NX);                       \
  else if (head_dim == 128) CEK_ROPE(T, 2, NX);                 \
  else CEK_ROPE(T, 4, NX);
  if (dtype == CEK_F16) {
    if (is_neox) { CEK_ROPE_E(__half, true) } else { CEK_ROPE_E(__half, false) }
  } else {
    if (is_neox) { CEK_ROPE_E(__nv_bfloat16, true) } else { CEK_ROPE_E(__nv_bfloat16, false) }
  }
#undef CEK_ROPE_E
#undef CEK_ROPE
  return s;
}

extern "C" int cek_quant_fp8_per_token(const void* a, void* aq, float* a_scale, int64_t M,
                                       int64_t K, int dtype, void* stream) {
  if (M < 0 || K <= 0 || K % 8 != 0 || K > 16384 || M > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (M == 0) return CEK_OK;
  if (!a || !aq || !a_scale) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(a) || (reinterpret_cast<uintptr_t>(aq) & 7u)) return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpt = (int)((K / 8 + 255) / 256);
  int s = CEK_OK;
#define CEK_QUANT(T, V)                                                                      \
  s = cek_host::launch_pdl(cek::quant_fp8_per_token_kernel<T, V>, dim3((unsigned)M), dim3(256), 0, st, a,  \
                           aq, a_scale, (int)K)
#define CEK_QUANT_V(T)                                                                       \
  if (vpt <= 1) CEK_QUANT(T, 1); else if (vpt <= 2) CEK_QUANT(T, 2);                         \
  else if (vpt <= 4) CEK_QUANT(T, 4); else CEK_QUANT(T, 8);
  if (dtype == CEK_F16) { CEK_QUANT_V(__half) } else { CEK_QUANT_V(__nv_bfloat16) }
#undef CEK_QUANT_V
#undef CEK_QUANT
  return s;
}
