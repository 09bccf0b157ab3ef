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
// Every lane's run of elements is contiguous, so with VEC each run (head
// values, gamma, cos and sin) moves as one vector access of E or 2E elements;
// without VEC (a pointer not 16-byte aligned) element by element.
template <typename T, int N>
struct __align__(sizeof(T) * N) Run { T v[N]; };
template <int N>
struct __align__(4 * N) RunF { float v[N]; };

template <int N, bool VEC, typename T>
__device__ __forceinline__ void load_run(const T* p, float* x) {
  if constexpr (VEC) {
    const Run<T, N> r = *reinterpret_cast<const Run<T, N>*>(p);
#pragma unroll
    for (int e = 0; e < N; ++e) x[e] = to_f32<T>(r.v[e]);
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) x[e] = to_f32<T>(p[e]);
  }
}
template <int N, bool VEC, typename T>
__device__ __forceinline__ void store_run(T* p, const float* x) {
  if constexpr (VEC) {
    Run<T, N> r;
#pragma unroll
    for (int e = 0; e < N; ++e) r.v[e] = from_f32<T>(x[e]);
    *reinterpret_cast<Run<T, N>*>(p) = r;
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) p[e] = from_f32<T>(x[e]);
  }
}
template <int N, bool VEC>
__device__ __forceinline__ void load_runf(const float* p, float* x) {
  if constexpr (VEC) {
    const RunF<N> r = *reinterpret_cast<const RunF<N>*>(p);
#pragma unroll
    for (int e = 0; e < N; ++e) x[e] = r.v[e];
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) x[e] = p[e];
  }
}

template <typename T, int E, bool NEOX, bool VEC>
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
  // the lane's two runs: [o0, o0 + E) and [o1, o1 + E) (adjacent when interleaved)
  const int o0 = NEOX ? lane * E : lane * 2 * E;
  const int o1 = NEOX ? D / 2 + lane * E : lane * 2 * E + E;

  float x[2 * E], g[2 * E], c[E], sn[E];
  if constexpr (NEOX) {
    load_run<E, VEC>(head + o0, x);
    load_run<E, VEC>(head + o1, x + E);
    load_run<E, VEC>(w + o0, g);
    load_run<E, VEC>(w + o1, g + E);
  } else {
    load_run<2 * E, VEC>(head + o0, x);
    load_run<2 * E, VEC>(w + o0, g);
  }
  load_runf<E, VEC>(cs + lane * E, c);
  load_runf<E, VEC>(cs + D / 2 + lane * E, sn);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) ss += x[e] * x[e];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int e = 0; e < 2 * E; ++e) x[e] = to_f32<T>(from_f32<T>(x[e] * inv * g[e]));
  float o[2 * E];
  if constexpr (NEOX) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o[e] = x[e] * c[e] - x[E + e] * sn[e];
      o[E + e] = x[E + e] * c[e] + x[e] * sn[e];
    }
    store_run<E, VEC>(head + o0, o);
    store_run<E, VEC>(head + o1, o + E);
  } else {
#pragma unroll
    for (int q = 0; q < E; ++q) {
      const float x0 = x[2 * q], x1 = x[2 * q + 1];
      o[2 * q] = x0 * c[q] - x1 * sn[q];
      o[2 * q + 1] = x1 * c[q] + x0 * sn[q];
    }
    store_run<2 * E, VEC>(head + o0, o);
  }
}

// ---- per-token dynamic e4m3 quantisation -------------------------------------
// s = max(amax, 1e-12) / 448 with IEEE division; q = e4m3_rn_sat(a / s).
// TPR threads per row (32..256), 256 / TPR rows per 256-thread CTA, VPT 16-byte
// vectors per thread (VPT <= 8); the grid is one resident wave that strides
// over the row groups.  The row stays in registers between the amax
// reduction and the quantisation, so it is read from HBM once.
//  * amax: an unsigned max over the 16-bit patterns with the sign bits
//    cleared (two lanes per instruction).  Non-negative fp16 / bf16 patterns
//    order as their values, and a NaN pattern sorts above infinity, so a row
//    holding a NaN gets a NaN amax and scale, as torch's amax gives.
//  * no clamp: the satfinite conversion saturates finite values beyond 448 to
//    +-448 and keeps NaN, which is what clamping to [-448, 448] first gives.
template <typename T, int TPR, int VPT>
__global__ void __launch_bounds__(256)
quant_fp8_per_token_kernel(const T* __restrict__ a, uint8_t* __restrict__ q, float* __restrict__ sc,
                           int M, int K) {
  constexpr int RPC = 256 / TPR, WPR = TPR / 32;
  __shared__ uint32_t sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const int r = threadIdx.x / TPR, t = threadIdx.x % TPR;
  const int nvec = K >> 3;
  const int groups = (M + RPC - 1) / RPC;
  for (int grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int m = grp * RPC + r;
    const bool live = m < M;
    const T* row = a + (size_t)(live ? m : 0) * K;
    uint4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = t + i * TPR;
      v[i] = (live && idx < nvec) ? __ldcs(reinterpret_cast<const uint4*>(row + idx * 8)) : make_uint4(0, 0, 0, 0);
    }
    uint32_t mx = 0;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      mx = __vmaxu2(mx, v[i].x & 0x7FFF7FFFu);
      mx = __vmaxu2(mx, v[i].y & 0x7FFF7FFFu);
      mx = __vmaxu2(mx, v[i].z & 0x7FFF7FFFu);
      mx = __vmaxu2(mx, v[i].w & 0x7FFF7FFFu);
    }
    uint32_t amax_bits = max(mx & 0xFFFFu, mx >> 16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax_bits = max(amax_bits, __shfl_xor_sync(0xffffffffu, amax_bits, o));
    if constexpr (WPR > 1) {
      if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = amax_bits;
      __syncthreads();
#pragma unroll
      for (int w = 0; w < WPR; ++w) amax_bits = max(amax_bits, sh[r * WPR + w]);
      __syncthreads();  // sh is rewritten by the next row group
    }
    if (!live) continue;
    const float amax = unpack2<T>(amax_bits).x;
    const float s = amax != amax ? amax : __fdiv_rn(fmaxf(amax, 1e-12f), 448.f);
    if (t == 0) sc[m] = s;
    // a / s correctly rounded without a division per element.  Markstein's
    // theorem ("IA-64 and Elementary Functions", 2000): if y is the correctly
    // rounded reciprocal of s and q is within one ulp of a / s, then
    // q + y * (a - s * q), the remainder exact by FMA and the sum rounded once,
    // is the correctly rounded quotient.  q0 = a * y can be 1.5 ulps off, so one
    // correction step first brings it within half an ulp (plus a term of order
    // 2^-24 ulp), and a second one rounds it correctly.  |a / s| <= 448, so no
    // quotient overflows; quotients too small for the theorem's normal range
    // round to e4m3 zero of the same sign either way.  A row whose scale is
    // not finite (an infinite or NaN input) takes the IEEE division, where the
    // remainder step would form 0 * inf.
    const float y = __frcp_rn(s);
    const bool exact_div = !isfinite(s);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = t + i * TPR;
      if (idx >= nvec) continue;
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack2<T>(w[j]);
        float2 rr;
        if (exact_div) {
          rr.x = __fdiv_rn(f.x, s);
          rr.y = __fdiv_rn(f.y, s);
        } else {
          float qx = __fmul_rn(f.x, y), qy = __fmul_rn(f.y, y);
          qx = __fmaf_rn(__fmaf_rn(-qx, s, f.x), y, qx);
          qy = __fmaf_rn(__fmaf_rn(-qy, s, f.y), y, qy);
          // s > 0, so the quotient has the sign of a; the correction steps
          // would turn a / s = -0 into +0 (a zero remainder added to -0)
          rr.x = copysignf(__fmaf_rn(__fmaf_rn(-qx, s, f.x), y, qx), f.x);
          rr.y = copysignf(__fmaf_rn(__fmaf_rn(-qy, s, f.y), y, qy), f.y);
        }
        const __nv_fp8x2_storage_t p2 = __nv_cvt_float2_to_fp8x2(rr, __NV_SATFINITE, __NV_E4M3);
        packed[j >> 1] |= (uint32_t)p2 << (16 * (j & 1));
      }
      *reinterpret_cast<uint2*>(q + (size_t)m * K + idx * 8) = make_uint2(packed[0], packed[1]);
    }
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
  const bool vec = cek_host::aligned16(qkv) && cek_host::aligned16(q_weight) && cek_host::aligned16(k_weight) &&
                   cek_host::aligned16(cos_sin_cache);
#define CEK_ROPE(T, E, NX)                                                                             \
  s = vec ? cek_host::launch_pdl(cek::qkv_norm_rope_kernel<T, E, NX, true>, grid, block, 0, st, qkv,       \
                                 positions, q_weight, k_weight, cos_sin_cache, m, hq, hkv, mp, eps)        \
          : cek_host::launch_pdl(cek::qkv_norm_rope_kernel<T, E, NX, false>, grid, block, 0, st, qkv,      \
                                 positions, q_weight, k_weight, cos_sin_cache, m, hq, hkv, mp, eps)
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
  // smallest row team whose per-thread share is at most 8 vectors (K <= 16384)
  const int64_t nvec = K / 8;
  const int tpr = nvec <= 256 ? 32 : nvec <= 512 ? 64 : nvec <= 1024 ? 128 : 256;
  const int vpt = (int)((nvec + tpr - 1) / tpr);
  const int rpc = 256 / tpr;
  const int64_t groups = (M + rpc - 1) / rpc;
  const int m = (int)M, k = (int)K;
  int s = CEK_OK;
  // one resident wave (the kernel strides over the row groups)
#define CEK_QUANT(T, TPR, V)                                                                          \
  do {                                                                                                \
    auto kern = cek::quant_fp8_per_token_kernel<T, TPR, V>;                                           \
    static const int per_sm = [&] {                                                                   \
      int b = 0;                                                                                      \
      return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, 256, 0) == cudaSuccess && b > 0 ? b \
                                                                                                  : 1; \
    }();                                                                                              \
    const dim3 grid((unsigned)std::min<int64_t>(groups, (int64_t)per_sm * cek_host::sm_count()));     \
    s = cek_host::launch_pdl(kern, grid, dim3(256), 0, st, a, aq, a_scale, m, k);                      \
  } while (0)
#define CEK_QUANT_V(T, TPR)                                                                       \
  if (vpt <= 1) CEK_QUANT(T, TPR, 1); else if (vpt <= 2) CEK_QUANT(T, TPR, 2);                    \
  else if (vpt <= 4) CEK_QUANT(T, TPR, 4); else CEK_QUANT(T, TPR, 8);
#define CEK_QUANT_T(T)                                                                            \
  if (tpr == 32) { CEK_QUANT_V(T, 32) } else if (tpr == 64) { CEK_QUANT_V(T, 64) }                \
  else if (tpr == 128) { CEK_QUANT_V(T, 128) } else { CEK_QUANT_V(T, 256) }
  if (dtype == CEK_F16) { CEK_QUANT_T(__half) } else { CEK_QUANT_T(__nv_bfloat16) }
#undef CEK_QUANT_T
#undef CEK_QUANT_V
#undef CEK_QUANT
  return s;
}
