// gemv_fp8.cu — FP8-weight GEMV / small-M GEMM for B200 (sm_100a).
//
// Computes y[m, n] = OutT( sum_k x[m, k] * deq(w[n, k]) * scale(n) ) for
// M up to 16 per M-tile (more M-tiles for larger M), the work of the
// reference's GEMV_fp8_pern_kernel / GEMV_fp8_pert_kernel
// (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:44-90, 322-368) and of its small-M
// GEMM regimes (csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:110-157, 2930-3139).
//
// Design (HBM-bound):
//  * Swap-AB tensor-core tiles.  A warp owns a 16-row group of W and a
//    K-slice.  W is the mma.sync m16n8k16 A operand (16 output channels x
//    16 k), the activations are the B operand (16 k x 8 tokens), fp32
//    accumulators.  Each FP8 pair is converted exactly to f16x2 / bf16x2 in
//    registers, so the dot product is the fp32 dequant-then-matmul of the
//    reference oracle up to fp32 summation order.  One conversion per two
//    weights and one MMA per 256 weights keep the SM ALUs far below the HBM
//    rate even at M = 16, where a scalar-FMA GEMV would be ALU-bound.
//  * K permutation.  Lane (g = lane/4, t = lane%4) loads 16 contiguous bytes
//    of rows g and g+8 at k = 64c + 16t and the 16 matching activations of
//    token g; the four 4-byte words feed four k16 MMA steps.  Any bijection
//    of k that is the same for A and B leaves the sum unchanged.
//  * Memory-level parallelism.  Each warp issues U = 4 chunk loads (2 x 16 B
//    per lane each) before consuming any; with 16 warps per CTA and several
//    CTAs per SM this keeps >40 KB per SM in flight.
//  * Split-K inside the CTA only (warps of one row group take disjoint
//    K-slices, reduced through shared memory in a fixed order): no global
//    scratch, no atomics, bit-reproducible results.
//  * PDL: weights never depend on the previous kernel, so the first batch of
//    weight loads is issued before griddepcontrol.wait; activation loads and
//    all stores come after it.
#include "gemv.cuh"
#include <type_traits>

namespace cek {

constexpr int kChunkK = 64;   // k per lane-quad load round (4 lanes x 16 B)
constexpr int kUnroll = 4;    // chunks in flight per warp
constexpr int kMaxWarps = 16;



template <typename InT, int FMT, int SCALE, typename OutT, int NT, bool FUSED>
__global__ void __launch_bounds__(kMaxWarps * 32)
gemv_fp8_kernel(const GemvParams p) {
  __shared__ float red[kMaxWarps][16][NT * 8];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cta = blockIdx.x / p.mtiles, mt = blockIdx.x % p.mtiles;
  const int rg_local = warp / p.ks, kslice = warp % p.ks;
  const int row0 = (cta * p.rg_per_cta + rg_local) * 16 + g;
  const int row1 = row0 + 8;
  const int tok_base = mt * NT * 8;
  const int nchunks = (p.K + kChunkK - 1) / kChunkK;
  const int cbeg = kslice * p.cpw;
  const int cend = min(cbeg + p.cpw, nchunks);
  const bool v0 = row0 < p.N, v1 = row1 < p.N;
  const uint8_t* w0 = p.w + (size_t)(v0 ? row0 : 0) * p.K + t * 16;
  const uint8_t* w1 = p.w + (size_t)(v1 ? row1 : 0) * p.K + t * 16;

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  bool waited = false;
  for (int c = cbeg; c < cend; c += kUnroll) {
    uint4 wa[kUnroll], wb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int kk = (c + u) * kChunkK + t * 16;
      const bool ok = (c + u < cend) && kk < p.K;
      wa[u] = (ok && v0) ? ldg_stream(w0 + (size_t)(c + u) * kChunkK) : make_uint4(0, 0, 0, 0);
      wb[u] = (ok && v1) ? ldg_stream(w1 + (size_t)(c + u) * kChunkK) : make_uint4(0, 0, 0, 0);
    }
    if (!waited) { pdl_wait(); waited = true; }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (c + u >= cend) break;
      const int kk = (c + u) * kChunkK + t * 16;
      uint32_t xw[NT][8];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = tok_base + j * 8 + g;
        if (tok < p.M && kk < p.K) {
          load_x16<InT, FUSED>(p, tok, kk, xw[j]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) xw[j][i] = 0u;
        }
      }
      const uint32_t wra[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
      const uint32_t wrb[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        uint32_t a[4];
        a[0] = cvt_pair<InT, FMT>(wra[s] & 0xFFFFu);
        a[1] = cvt_pair<InT, FMT>(wrb[s] & 0xFFFFu);
        a[2] = cvt_pair<InT, FMT>(wra[s] >> 16);
        a[3] = cvt_pair<InT, FMT>(wrb[s] >> 16);
#pragma unroll
        for (int j = 0; j < NT; ++j) mma16816<InT>(acc[j], a, xw[j][2 * s], xw[j][2 * s + 1]);
      }
    }
  }
  if (!waited) pdl_wait();

  // Cross-warp (split-K) reduction in a fixed order.
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    red[warp][g][j * 8 + 2 * t] = acc[j][0];
    red[warp][g][j * 8 + 2 * t + 1] = acc[j][1];
    red[warp][g + 8][j * 8 + 2 * t] = acc[j][2];
    red[warp][g + 8][j * 8 + 2 * t + 1] = acc[j][3];
  }
  __syncthreads();
  const int rows_cta = p.rg_per_cta * 16;
  const int entries = rows_cta * NT * 8;
  for (int e = threadIdx.x; e < entries; e += blockDim.x) {
    const int tl = e / rows_cta, rr = e % rows_cta;
    const int tok = tok_base + tl;
    const int n = cta * rows_cta + rr;
    if (tok >= p.M || n >= p.N) continue;
    const int rgl = rr >> 4, r = rr & 15;
    float s = 0.f;
    for (int q = 0; q < p.ks; ++q) s += red[rgl * p.ks + q][r][tl];
    s *= load_scale<SCALE>(p.scale, n);
    reinterpret_cast<OutT*>(p.y)[(size_t)tok * p.N + n] = from_f32<OutT>(s);
  }
}

// ---- host side --------------------------------------------------------------

struct GemvLaunch { int ks, rg_per_cta, warps, cpw, mtiles, nt; int64_t ctas; };

// Split-K / CTA shape heuristic.  Goal: about 32 resident warps per SM on all
// 148 SMs with every warp owning at least one U-deep batch of chunk loads.
static GemvLaunch plan_gemv(int64_t M, int64_t N, int64_t K) {
  GemvLaunch L;
  const int64_t rgs = (N + 15) / 16;
  const int64_t nchunks = (K + kChunkK - 1) / kChunkK;
  const int64_t target_warps = 148 * 32;
  int ks = 1;
  while (ks < 16 && rgs * ks < target_warps && nchunks >= (int64_t)(ks * 2) * kUnroll) ks *= 2;
  L.ks = ks;
  L.warps = ks >= 8 ? ks : 8;
  L.rg_per_cta = L.warps / ks;
  L.cpw = (int)((nchunks + ks - 1) / ks);
  L.nt = M <= 8 ? 1 : 2;
  L.mtiles = (int)((M + 8 * L.nt - 1) / (8 * L.nt));
  L.ctas = ((rgs + L.rg_per_cta - 1) / L.rg_per_cta) * L.mtiles;
  return L;
}

template <typename InT, int FMT, int SCALE, typename OutT, int NT, bool FUSED>
static int launch_one(const GemvParams& p, const GemvLaunch& L, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)L.ctas);
  cfg.blockDim = dim3(L.warps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_fp8_kernel<InT, FMT, SCALE, OutT, NT, FUSED>, p);
  return e == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

template <typename InT, int FMT, int SCALE, typename OutT, bool FUSED>
static int dispatch_nt(const GemvParams& p, const GemvLaunch& L, cudaStream_t st) {
  return L.nt == 1 ? launch_one<InT, FMT, SCALE, OutT, 1, FUSED>(p, L, st)
                   : launch_one<InT, FMT, SCALE, OutT, 2, FUSED>(p, L, st);
}

template <typename InT, typename OutT, bool FUSED>
static int dispatch_fmt_scale(const GemvParams& p, const GemvLaunch& L, int w_fmt, int scale_kind,
                              cudaStream_t st) {
#define CEK_CASE(F, S)                                                   \
  if (w_fmt == F && scale_kind == S) return dispatch_nt<InT, F, S, OutT, FUSED>(p, L, st);
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERN_F16)
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERN_F32)
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERT_F32)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERN_F16)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERN_F32)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERT_F32)
#undef CEK_CASE
  return CEK_ERR_INVALID_ARG;
}

int gemv_launch(const GemvParams& base, int x_dtype, int y_dtype, int w_fmt, int scale_kind,
                bool fused, cudaStream_t st) {
  GemvLaunch L = plan_gemv(base.M, base.N, base.K);
  GemvParams p = base;
  p.ks = L.ks; p.rg_per_cta = L.rg_per_cta; p.mtiles = L.mtiles; p.cpw = L.cpw;
  if (fused) {
    if (x_dtype != y_dtype) return CEK_ERR_INVALID_ARG;
    if (x_dtype == CEK_F16) return dispatch_fmt_scale<__half, __half, true>(p, L, w_fmt, scale_kind, st);
    return dispatch_fmt_scale<__nv_bfloat16, __nv_bfloat16, true>(p, L, w_fmt, scale_kind, st);
  }
  if (x_dtype == CEK_F16 && y_dtype == CEK_F16)
    return dispatch_fmt_scale<__half, __half, false>(p, L, w_fmt, scale_kind, st);
  if (x_dtype == CEK_F16 && y_dtype == CEK_BF16)
    return dispatch_fmt_scale<__half, __nv_bfloat16, false>(p, L, w_fmt, scale_kind, st);
  if (x_dtype == CEK_BF16 && y_dtype == CEK_F16)
    return dispatch_fmt_scale<__nv_bfloat16, __half, false>(p, L, w_fmt, scale_kind, st);
  return dispatch_fmt_scale<__nv_bfloat16, __nv_bfloat16, false>(p, L, w_fmt, scale_kind, st);
}

int gemv_run(const GemvParams& base, int x_dtype, int y_dtype, int w_fmt, int scale_kind, bool fused,
             void* workspace, int64_t ws_bytes, cudaStream_t st) {
  if (workspace && base.M <= 16 && ws_bytes >= gemv_streamk_workspace_bytes(base.M, base.N, base.K))
    return gemv_streamk_launch(base, x_dtype, y_dtype, w_fmt, scale_kind, fused, workspace, ws_bytes, st);
  return gemv_launch(base, x_dtype, y_dtype, w_fmt, scale_kind, fused, st);
}

}  // namespace cek

extern "C" int64_t cek_gemv_fp8_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return cek::gemv_streamk_workspace_bytes(M, N, K);
}

extern "C" int cek_gemv_fp8(const void* x, const void* w, const void* scale, void* y, int64_t M,
                            int64_t N, int64_t K, int x_dtype, int y_dtype, int w_fmt,
                            int scale_kind, void* workspace, int64_t workspace_bytes,
                            void* stream) {
  using namespace cek_host;
  if (M < 0 || N < 0 || K < 0 || workspace_bytes < 0) return CEK_ERR_INVALID_ARG;
  if ((x_dtype != CEK_F16 && x_dtype != CEK_BF16) || (y_dtype != CEK_F16 && y_dtype != CEK_BF16))
    return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CEK_OK;
  if (K % 16 != 0 || N > INT32_MAX || K > INT32_MAX || M > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if (!x || !w || !scale || !y) return CEK_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w) || (workspace && !aligned16(workspace))) return CEK_ERR_ALIGNMENT;
  cek::GemvParams p = {};
  p.x = x; p.w = static_cast<const uint8_t*>(w); p.scale = scale; p.y = y;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  return cek::gemv_run(p, x_dtype, y_dtype, w_fmt, scale_kind, false, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}
