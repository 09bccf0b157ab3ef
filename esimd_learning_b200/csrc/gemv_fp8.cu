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
//  * Memory-level parallelism.  Each warp keeps two batches of U = 2 chunks
//    (weights and the matching activations) in flight: the loads of batch
//    b+1 are issued before batch b is converted and multiplied.  8-warp CTAs,
//    ~48 warps per SM over the grid.
//  * Split-K inside the CTA only (warps of one row group take disjoint
//    K-slices, reduced through shared memory in a fixed order): no global
//    scratch, no atomics, bit-reproducible results.
//  * PDL: with `early_weights` set (the preceding kernel does not write W)
//    the first batch of weight loads is issued before griddepcontrol.wait;
//    activation loads and all stores always come after it.
#include "gemv.cuh"
#include <algorithm>
#include <cstdlib>
#include <type_traits>

namespace cek {

constexpr int kChunkK = 64;   // k per lane-quad load round (4 lanes x 16 B)
constexpr int kMaxWarps = 16; // warps per CTA: max(8, ks)

// Chunks per batch (two batches in flight per warp): 2 for one token tile,
// 1 for two (their activation registers double).
#ifndef CEK_GEMV_U1
#define CEK_GEMV_U1 2
#endif
template <int NT> struct UnrollOf { static constexpr int value = NT == 1 ? CEK_GEMV_U1 : 1; };

// Weight stream load (16 B, read once: no L1 allocation).
CEK_DEVICE uint4 ldg_w(const void* p) {
  uint4 r;
#if CEK_GEMV_WLOAD == 1
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
#elif CEK_GEMV_WLOAD == 2
  asm volatile("ld.global.nc.L1::no_allocate.L2::128B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
#elif CEK_GEMV_WLOAD == 3
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
#else
  r = ldg_stream(p);
#endif
  return r;
}

// One batch: U chunks of 16 rows x 64 k of W for this warp's lanes, plus the
// matching activations of the warp's NT token tiles.
template <int NT>
struct Batch {
  static constexpr int U = UnrollOf<NT>::value;
  uint4 wa[U], wb[U];
  uint32_t xw[U][NT][8];
};

template <int NT>
struct WarpCtx {
  const uint8_t* w0;
  const uint8_t* w1;
  bool v0, v1;
  int g, t, tok_base, cend;
};

template <int NT>
CEK_DEVICE void issue_w(const GemvParams& p, const WarpCtx<NT>& c, int ch, Batch<NT>& b) {
#pragma unroll
  for (int u = 0; u < Batch<NT>::U; ++u) {
    const int kk = (ch + u) * kChunkK + c.t * 16;
    const bool ok = (ch + u < c.cend) && kk < p.K;
    b.wa[u] = (ok && c.v0) ? ldg_w(c.w0 + (size_t)(ch + u) * kChunkK) : make_uint4(0, 0, 0, 0);
    b.wb[u] = (ok && c.v1) ? ldg_w(c.w1 + (size_t)(ch + u) * kChunkK) : make_uint4(0, 0, 0, 0);
  }
}

template <typename InT, bool FUSED, int NT>
CEK_DEVICE void issue_x(const GemvParams& p, const WarpCtx<NT>& c, int ch, Batch<NT>& b) {
#pragma unroll
  for (int u = 0; u < Batch<NT>::U; ++u) {
    const int kk = (ch + u) * kChunkK + c.t * 16;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int tok = c.tok_base + j * 8 + c.g;
      if (ch + u < c.cend && tok < p.M && kk < p.K) {
        load_x16<InT, FUSED>(p, tok, kk, b.xw[u][j]);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) b.xw[u][j][i] = 0u;
      }
    }
  }
}

template <typename InT, int FMT, int NT>
CEK_DEVICE void consume(const Batch<NT>& b, float (&acc)[NT][4]) {
#pragma unroll
  for (int u = 0; u < Batch<NT>::U; ++u) {
    const uint32_t wra[4] = {b.wa[u].x, b.wa[u].y, b.wa[u].z, b.wa[u].w};
    const uint32_t wrb[4] = {b.wb[u].x, b.wb[u].y, b.wb[u].z, b.wb[u].w};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t a[4];
      a[0] = cvt_pair<InT, FMT>(wra[s] & 0xFFFFu);
      a[1] = cvt_pair<InT, FMT>(wrb[s] & 0xFFFFu);
      a[2] = cvt_pair<InT, FMT>(wra[s] >> 16);
      a[3] = cvt_pair<InT, FMT>(wrb[s] >> 16);
#pragma unroll
      for (int j = 0; j < NT; ++j) mma16816<InT>(acc[j], a, b.xw[u][j][2 * s], b.xw[u][j][2 * s + 1]);
    }
  }
}

// PUSH: the tensor-parallel push epilogues (all-reduce slots or all-gather
// rows over peer memory) instead of the local store; a separate
// instantiation, so the plain kernel carries no trace of them.
template <typename InT, int FMT, int SCALE, typename OutT, int NT, bool FUSED, bool PUSH = false>
__global__ void __launch_bounds__(kMaxWarps * 32)
gemv_fp8_kernel(const __grid_constant__ GemvParams p) {
  constexpr int U = Batch<NT>::U;
  __shared__ float red[kMaxWarps][16][NT * 8];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The parameters stay in parameter space (no per-thread copy); a
  // multi-GEMV CTA overrides its matrix's pointers and row count here.
  int cta = blockIdx.x / p.mtiles;
  const int mt = blockIdx.x % p.mtiles;
  const uint8_t* pw = p.w;
  const void* pscale = p.scale;
  void* py = p.y;
  int pN = p.N;
  if (p.nmat > 0) {  // multi-GEMV: pick this CTA's matrix
    int m = 0;
    while (m + 1 < p.nmat && cta >= p.mcta_off[m + 1]) ++m;
    pw = p.mws[m];
    pscale = p.mscales[m];
    py = p.mys[m];
    pN = p.mns[m];
    cta -= p.mcta_off[m];
  }
  const int rg_local = warp / p.ks, kslice = warp % p.ks;
  WarpCtx<NT> c;
  c.g = lane >> 2;
  c.t = lane & 3;
  const int row0 = (cta * p.rg_per_cta + rg_local) * 16 + c.g;
  const int row1 = row0 + 8;
  c.tok_base = mt * NT * 8;
  const int nchunks = (p.K + kChunkK - 1) / kChunkK;
  const int cbeg = kslice * p.cpw;
  c.cend = min(cbeg + p.cpw, nchunks);
  c.v0 = row0 < pN;
  c.v1 = row1 < pN;
  c.w0 = pw + (size_t)(c.v0 ? row0 : 0) * p.K + c.t * 16;
  c.w1 = pw + (size_t)(c.v1 ? row1 : 0) * p.K + c.t * 16;

  // No early griddepcontrol.launch_dependents here: the kernel that follows
  // is often the persistent bulk GEMV (one 220 KB CTA per SM), whose CTAs,
  // launched early, would take whole SMs from this grid's last wave while
  // they wait (measured: the chain's down projection at M = 16 ran 80 us
  // alone and far longer in the graph).  The dependent grid launches when
  // this one completes.

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  // Two batches in flight: while one is converted and multiplied, the loads
  // of the next are outstanding.
  Batch<NT> A, B;
  if (p.early_weights) {
    issue_w(p, c, cbeg, A);
    pdl_wait();
  } else {
    pdl_wait();
    issue_w(p, c, cbeg, A);
  }
  issue_x<InT, FUSED>(p, c, cbeg, A);
  for (int ch = cbeg; ch < c.cend; ch += 2 * U) {
    issue_w(p, c, ch + U, B);
    issue_x<InT, FUSED>(p, c, ch + U, B);
    consume<InT, FMT>(A, acc);
    if (ch + U >= c.cend) break;
    issue_w(p, c, ch + 2 * U, A);
    issue_x<InT, FUSED>(p, c, ch + 2 * U, A);
    consume<InT, FMT>(B, acc);
  }

  // Cross-warp (split-K) reduction in a fixed order.
  const int g = c.g, t = c.t;
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
    const int tok = c.tok_base + tl;
    const int n = cta * rows_cta + rr;
    if (tok >= p.M || n >= pN) continue;
    const int rgl = rr >> 4, r = rr & 15;
    float s = 0.f;
    for (int q = 0; q < p.ks; ++q) s += red[rgl * p.ks + q][r][tl];
    s *= load_scale<SCALE>(pscale, n);
    if constexpr (!PUSH)
      reinterpret_cast<OutT*>(py)[(size_t)tok * pN + n] = from_f32<OutT>(s);
    else
      store_out_push<OutT>(p.ar_peers, p.ar_sync, p.ar_rank, p.ar_world, p.ag_off, p.ag_n, p.ag_row0, p.M, p.N, tok,
                           n, from_f32<OutT>(s));
  }
}

// ---- host side --------------------------------------------------------------

struct GemvLaunch { int ks, rg_per_cta, warps, cpw, mtiles, nt; int64_t ctas; };

// Split-K / CTA shape.  ks warps share one 16-row group (disjoint K-slices);
// a CTA is max(8, ks) warps holding max(8, ks)/ks row groups.  ks grows
// (up to 16) while the grid has fewer than ~48 warps per SM and every warp
// keeps at least one pair of batches.  CEK_GEMV_KS overrides ks (tuning).
static GemvLaunch plan_gemv(int64_t M, int64_t N, int64_t K) {
  GemvLaunch L;
  const int64_t rgs = (N + 15) / 16;
  const int64_t nchunks = (K + kChunkK - 1) / kChunkK;
  const int64_t target_warps = 148 * 48;
  int ks = 1;
  const int U = M <= 8 ? UnrollOf<1>::value : UnrollOf<2>::value;
  while (ks < kMaxWarps && rgs * ks < target_warps && nchunks >= (int64_t)(ks * 2) * 2 * U) ks *= 2;
  static const int ks_env = [] {
    const char* v = std::getenv("CEK_GEMV_KS");
    return v ? std::atoi(v) : 0;
  }();
  if (ks_env == 1 || ks_env == 2 || ks_env == 4 || ks_env == 8 || ks_env == 16) ks = ks_env;
  L.ks = ks;
  L.warps = ks > 8 ? ks : 8;
  static const int warps_env = [] {
    const char* v = std::getenv("CEK_GEMV_WARPS");
    return v ? std::atoi(v) : 0;
  }();
  if (warps_env == 8 || warps_env == 16) L.warps = warps_env > ks ? warps_env : ks;
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
  // Programmatic launch only behind the fused op's stats kernel (a few CTAs).
  // Behind the persistent bulk GEMV it measured slower: the chain at M = 16
  // (down projection here) took 311 us per layer with it, 209 us without.
  attr[0].val.programmaticStreamSerializationAllowed = (cek_host::pdl_enabled() && FUSED) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = p.ar_world > 0 ? cudaLaunchKernelEx(&cfg, gemv_fp8_kernel<InT, FMT, SCALE, OutT, NT, FUSED, true>, p)
                                  : cudaLaunchKernelEx(&cfg, gemv_fp8_kernel<InT, FMT, SCALE, OutT, NT, FUSED, false>, p);
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
  if (!fused) {
    const int s = gemv_bulk_launch(base, x_dtype, y_dtype, w_fmt, scale_kind, st);
    if (s != CEK_ERR_UNSUPPORTED || base.y_gelu) return s;  // only the bulk kernel forms gelu(gate) * up
  }
  GemvLaunch L = plan_gemv(base.M, base.N, base.K);  // multi-GEMV: N = sum of the matrices' N
  GemvParams p = base;
  p.ks = L.ks; p.rg_per_cta = L.rg_per_cta; p.mtiles = L.mtiles; p.cpw = L.cpw;
  if (p.nmat > 0) {
    int64_t ctas = 0;
    for (int m = 0; m < p.nmat; ++m) {
      p.mcta_off[m] = (int)ctas;
      ctas += ((int64_t)(p.mns[m] + 15) / 16 + L.rg_per_cta - 1) / L.rg_per_cta;
    }
    p.mcta_off[p.nmat] = (int)ctas;
    L.ctas = ctas * L.mtiles;
  }
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

}  // namespace cek

extern "C" int cek_gemv_fp8(const void* x, const void* w, const void* scale, void* y, int64_t M,
                            int64_t N, int64_t K, int x_dtype, int y_dtype, int w_fmt,
                            int scale_kind, unsigned flags, void* stream) {
  using namespace cek_host;
  if (M < 0 || N < 0 || K < 0) return CEK_ERR_INVALID_ARG;
  if ((x_dtype != CEK_F16 && x_dtype != CEK_BF16) || (y_dtype != CEK_F16 && y_dtype != CEK_BF16))
    return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (flags & ~(unsigned)(CEK_GEMV_EARLY_WEIGHTS | CEK_GEMV_GELU_MUL_OUTPUT)) return CEK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CEK_OK;
  if (K % 16 != 0 || N > INT32_MAX || K > INT32_MAX || M > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if (!x || !w || !scale || !y) return CEK_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w)) return CEK_ERR_ALIGNMENT;
  cek::GemvParams p = {};
  p.x = x; p.w = static_cast<const uint8_t*>(w); p.scale = scale; p.y = y;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.early_weights = (flags & CEK_GEMV_EARLY_WEIGHTS) ? 1 : 0;
  p.y_gelu = (flags & CEK_GEMV_GELU_MUL_OUTPUT) ? 1 : 0;
  return cek::gemv_launch(p, x_dtype, y_dtype, w_fmt, scale_kind, false,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int cek_gemv_fp8_multi(const void* x, const void* const* ws, const void* const* scales,
                                  void* const* ys, const int64_t* Ns, int count, int64_t M, int64_t K,
                                  int x_dtype, int y_dtype, int w_fmt, int scale_kind, unsigned flags,
                                  void* stream) {
  using namespace cek_host;
  if (count < 1 || count > cek::kMaxMats || !ws || !scales || !ys || !Ns) return CEK_ERR_INVALID_ARG;
  if (M < 0 || K < 0 || K % 16 != 0 || M > INT32_MAX || K > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if ((x_dtype != CEK_F16 && x_dtype != CEK_BF16) || (y_dtype != CEK_F16 && y_dtype != CEK_BF16))
    return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (flags & ~(unsigned)CEK_GEMV_EARLY_WEIGHTS) return CEK_ERR_INVALID_ARG;
  if (!x) return CEK_ERR_INVALID_ARG;
  int64_t total = 0;
  for (int m = 0; m < count; ++m) {
    if (Ns[m] <= 0 || Ns[m] > INT32_MAX || !ws[m] || !scales[m] || !ys[m]) return CEK_ERR_INVALID_ARG;
    if (!aligned16(ws[m])) return CEK_ERR_ALIGNMENT;
    total += Ns[m];
  }
  if (M == 0) return CEK_OK;
  if (!aligned16(x)) return CEK_ERR_ALIGNMENT;
  cek::GemvParams p = {};
  p.x = x;
  p.M = (int)M; p.N = (int)std::min<int64_t>(total, INT32_MAX); p.K = (int)K;
  p.early_weights = (flags & CEK_GEMV_EARLY_WEIGHTS) ? 1 : 0;
  p.nmat = count;
  for (int m = 0; m < count; ++m) {
    p.mws[m] = static_cast<const uint8_t*>(ws[m]);
    p.mscales[m] = scales[m];
    p.mys[m] = ys[m];
    p.mns[m] = (int)Ns[m];
  }
  p.w = p.mws[0]; p.scale = p.mscales[0]; p.y = p.mys[0];
  return cek::gemv_launch(p, x_dtype, y_dtype, w_fmt, scale_kind, false, static_cast<cudaStream_t>(stream));
}
