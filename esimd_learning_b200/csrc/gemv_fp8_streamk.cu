// gemv_fp8_streamk.cu — persistent, TMA-fed, stream-K FP8 GEMV (M <= 16).
//
// Same arithmetic as gemv_fp8.cu (exact FP8 -> 16-bit conversion in
// registers, mma.sync m16n8k16 swap-AB tiles with fp32 accumulators, scale in
// the epilogue), different data movement:
//
//  * Work units.  W is cut into units of 32 rows (two 16-row groups, a
//    "pair") x KC bytes of K.  The units are ordered pair-major and split
//    into gridDim.x equal contiguous ranges, one per CTA, with one CTA per
//    SM (stream-K): every SM streams the same number of weight bytes, so
//    there is no wave tail whatever N and K are.
//  * Producer warp.  One elected lane streams the CTA's units into a
//    STAGES-deep shared-memory ring with 1-D bulk copies
//    (cp.async.bulk, one per row, KC contiguous bytes each), completion
//    tracked by transaction-count mbarriers.  It runs ahead of the math by
//    up to STAGES units (~170 KB per SM in flight), independent of the
//    consumers' progress.  Weights never depend on the previous kernel, so it
//    starts before griddepcontrol.wait (PDL).
//  * Consumer warps (8).  Warp w takes the KC/8-byte K-slice w of each unit
//    for both row groups, reads its fragments from shared memory (rows padded
//    by 64 B so the 16-byte reads are bank-conflict free), loads the matching
//    activations from global/L1 and issues the MMAs.  When the CTA reaches
//    the end of a pair (or of its range) the 8 slices are reduced through
//    shared memory in a fixed order.
//  * Fixup.  A pair whose units span several CTAs is finished by the last CTA
//    to arrive: each contributor stores its fp32 partial into its slot of the
//    workspace, fences, and increments the pair's counter; the CTA that sees
//    the final count sums the slots in slot order (bit-reproducible), applies
//    the scale, writes y, and resets the counter to zero for the next call.
//    No CTA ever waits for another CTA.
//  * Bounded waits.  Every mbarrier wait gives up after a fixed number of
//    polls; a consumer that gives up writes NaN into the outputs of the pairs
//    it had not finished and exits, so a failure is visible and the context
//    stays usable.
#include "gemv.cuh"
#include <algorithm>

namespace cek {

namespace sk {

constexpr int kRows = 32;
constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kWaitPolls = 1 << 22;

template <int KC>
struct Cfg {
  static constexpr int kPitch = KC + 64;                 // smem row pitch
  static constexpr int kStageBytes = kRows * kPitch;
  static constexpr int kSub = KC / kConsumers;           // bytes of K per consumer per unit
  static constexpr int kChunks = kSub / 64;
  static_assert(kSub % 64 == 0, "consumer slice must hold whole 64-byte chunks");
};

CEK_DEVICE uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
CEK_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
CEK_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
CEK_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (int i = 0; i < kWaitPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
CEK_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
CEK_DEVICE void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
CEK_DEVICE void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
CEK_DEVICE void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

CEK_DEVICE int64_t range_start(int64_t c, int64_t T, int64_t G) { return c * T / G; }
CEK_DEVICE int owner(int64_t u, int64_t T, int G) {
  int64_t c = u * G / T;
  while (c + 1 < G && range_start(c + 1, T, G) <= u) ++c;
  while (c > 0 && range_start(c, T, G) > u) --c;
  return (int)c;
}

}  // namespace sk

template <typename InT, int FMT, int SCALE, typename OutT, int NT, bool FUSED, int KC, int STAGES>
__global__ void __launch_bounds__(sk::kThreads, 1)
gemv_fp8_streamk_kernel(const GemvParams p) {
  using C = sk::Cfg<KC>;
  constexpr int MT = NT * 8;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + STAGES * C::kStageBytes);  // [8][32][MT]
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t T = (int64_t)p.pairs * p.uk;
  const int G = gridDim.x;
  const int64_t u0 = sk::range_start(blockIdx.x, T, G);
  const int64_t u1 = sk::range_start(blockIdx.x + 1, T, G);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sk::mbar_init(sk::smem_addr(&full_bar[s]), 1);
      sk::mbar_init(sk::smem_addr(&empty_bar[s]), sk::kConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int i = 0;
      for (int64_t u = u0; u < u1; ++u, ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !sk::mbar_wait(sk::smem_addr(&empty_bar[s]), ((i / STAGES) - 1) & 1)) return;
        const int pair = (int)(u / p.uk), kt = (int)(u % p.uk);
        const int row0 = pair * sk::kRows;
        const int rows = min(sk::kRows, p.N - row0);
        const int k0 = kt * KC;
        const int kb = min(KC, p.K - k0);
        const uint32_t bar = sk::smem_addr(&full_bar[s]);
        sk::mbar_expect_tx(bar, (uint32_t)(rows * kb));
        uint8_t* stage = smem + s * C::kStageBytes;
        const uint8_t* src = p.w + (size_t)row0 * p.K + k0;
        for (int r = 0; r < rows; ++r)
          sk::bulk_g2s(sk::smem_addr(stage + r * C::kPitch), src + (size_t)r * p.K, (uint32_t)kb, bar);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  const int g = lane >> 2, t = lane & 3;
  float acc[2][NT][4];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[r][j][0] = acc[r][j][1] = acc[r][j][2] = acc[r][j][3] = 0.f;

  int i = 0;
  for (int64_t u = u0; u < u1; ++u, ++i) {
    const int s = i % STAGES;
    const int pair = (int)(u / p.uk), kt = (int)(u % p.uk);
    if (!sk::mbar_wait(sk::smem_addr(&full_bar[s]), (i / STAGES) & 1)) {
      // give up: poison the outputs this CTA still owed, then leave
      const int plast = (int)((u1 - 1) / p.uk);
      for (int pp = pair; pp <= plast; ++pp)
        for (int e = ctid; e < sk::kRows * MT; e += sk::kConsumers * 32) {
          const int tok = e / sk::kRows, n = pp * sk::kRows + e % sk::kRows;
          if (tok < p.M && n < p.N)
            reinterpret_cast<OutT*>(p.y)[(size_t)tok * p.N + n] = from_f32<OutT>(__int_as_float(0x7fc00000));
        }
      return;
    }
    const uint8_t* stage = smem + s * C::kStageBytes;
#pragma unroll
    for (int ch = 0; ch < C::kChunks; ++ch) {
      const int koff = cw * C::kSub + ch * 64 + t * 16;  // byte offset inside the unit
      const int kk = kt * KC + koff;
      const bool kv = kk < p.K;
      uint4 wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // rows g, g+8, 16+g, 24+g
        const int r = (q >> 1) * 16 + (q & 1) * 8 + g;
        wv[q] = kv ? *reinterpret_cast<const uint4*>(stage + r * C::kPitch + koff) : make_uint4(0, 0, 0, 0);
      }
      uint32_t xw[NT][8];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const int tok = j * 8 + g;
        if (tok < p.M && kv) {
          load_x16<InT, FUSED>(p, tok, kk, xw[j]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) xw[j][e] = 0u;
        }
      }
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const uint32_t w0[4] = {wv[0].x, wv[0].y, wv[0].z, wv[0].w};
        const uint32_t w1[4] = {wv[1].x, wv[1].y, wv[1].z, wv[1].w};
        const uint32_t w2[4] = {wv[2].x, wv[2].y, wv[2].z, wv[2].w};
        const uint32_t w3[4] = {wv[3].x, wv[3].y, wv[3].z, wv[3].w};
        uint32_t a0[4], a1[4];
        a0[0] = cvt_pair<InT, FMT>(w0[st] & 0xFFFFu);
        a0[1] = cvt_pair<InT, FMT>(w1[st] & 0xFFFFu);
        a0[2] = cvt_pair<InT, FMT>(w0[st] >> 16);
        a0[3] = cvt_pair<InT, FMT>(w1[st] >> 16);
        a1[0] = cvt_pair<InT, FMT>(w2[st] & 0xFFFFu);
        a1[1] = cvt_pair<InT, FMT>(w3[st] & 0xFFFFu);
        a1[2] = cvt_pair<InT, FMT>(w2[st] >> 16);
        a1[3] = cvt_pair<InT, FMT>(w3[st] >> 16);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          mma16816<InT>(acc[0][j], a0, xw[j][2 * st], xw[j][2 * st + 1]);
          mma16816<InT>(acc[1][j], a1, xw[j][2 * st], xw[j][2 * st + 1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) sk::mbar_arrive(sk::smem_addr(&empty_bar[s]));

    if (kt != p.uk - 1 && u != u1 - 1) continue;

    // ---- end of this CTA's share of `pair`: reduce the 8 K-slices ----
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        float* rb = red + (size_t)cw * sk::kRows * MT;
        rb[(r * 16 + g) * MT + j * 8 + 2 * t] = acc[r][j][0];
        rb[(r * 16 + g) * MT + j * 8 + 2 * t + 1] = acc[r][j][1];
        rb[(r * 16 + g + 8) * MT + j * 8 + 2 * t] = acc[r][j][2];
        rb[(r * 16 + g + 8) * MT + j * 8 + 2 * t + 1] = acc[r][j][3];
        acc[r][j][0] = acc[r][j][1] = acc[r][j][2] = acc[r][j][3] = 0.f;
      }
    sk::consumer_sync();
    const int64_t pu0 = (int64_t)pair * p.uk, pu1 = pu0 + p.uk;
    OutT* y = reinterpret_cast<OutT*>(p.y);
    if (pu0 >= u0 && pu1 <= u1) {
      for (int e = ctid; e < sk::kRows * MT; e += sk::kConsumers * 32) {
        const int tok = e / sk::kRows, r = e % sk::kRows, n = pair * sk::kRows + r;
        if (tok >= p.M || n >= p.N) continue;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < sk::kConsumers; ++q) v += red[((size_t)q * sk::kRows + r) * MT + tok];
        y[(size_t)tok * p.N + n] = from_f32<OutT>(v * load_scale<SCALE>(p.scale, n));
      }
    } else {
      const int c0 = sk::owner(pu0, T, G), c1 = sk::owner(pu1 - 1, T, G);
      const int ncontrib = c1 - c0 + 1, slot = blockIdx.x - c0;
      float* part = p.partials + ((size_t)pair * p.max_contrib + slot) * sk::kRows * MT;
      for (int e = ctid; e < sk::kRows * MT; e += sk::kConsumers * 32) {
        const int tok = e / sk::kRows, r = e % sk::kRows;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < sk::kConsumers; ++q) v += red[((size_t)q * sk::kRows + r) * MT + tok];
        part[e] = v;
      }
      __threadfence();
      sk::consumer_sync();
      if (ctid == 0) s_last = atomicAdd(&p.counters[pair], 1) == ncontrib - 1;
      sk::consumer_sync();
      if (s_last) {
        __threadfence();
        const float* base = p.partials + (size_t)pair * p.max_contrib * sk::kRows * MT;
        for (int e = ctid; e < sk::kRows * MT; e += sk::kConsumers * 32) {
          const int tok = e / sk::kRows, r = e % sk::kRows, n = pair * sk::kRows + r;
          if (tok >= p.M || n >= p.N) continue;
          float v = 0.f;
          for (int q = 0; q < ncontrib; ++q) v += __ldcg(base + (size_t)q * sk::kRows * MT + e);
          y[(size_t)tok * p.N + n] = from_f32<OutT>(v * load_scale<SCALE>(p.scale, n));
        }
        if (ctid == 0) p.counters[pair] = 0;
      }
    }
    sk::consumer_sync();
  }
}

// ---- host side ------------------------------------------------------------------

namespace sk_host {

constexpr int kKC = 1024;
constexpr int kStages = 5;

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

struct Plan { int pairs, uk, G, max_contrib, nt; int64_t T, ws_bytes, counters_bytes; };

Plan plan(int64_t M, int64_t N, int64_t K, int sms) {
  Plan P;
  P.pairs = (int)((N + sk::kRows - 1) / sk::kRows);
  P.uk = (int)((K + kKC - 1) / kKC);
  P.T = (int64_t)P.pairs * P.uk;
  P.G = (int)std::min<int64_t>(P.T, sms);
  P.nt = M <= 8 ? 1 : 2;
  int mc = 1;
  for (int pr = 0; pr < P.pairs; ++pr) {
    const int64_t a = (int64_t)pr * P.uk, b = a + P.uk - 1;
    const int64_t ca = a * P.G / P.T, cb = b * P.G / P.T;  // owners up to +-1
    mc = std::max<int>(mc, (int)(cb - ca + 3));
  }
  P.max_contrib = std::min(mc, P.uk);
  P.counters_bytes = ((int64_t)P.pairs * 4 + 255) / 256 * 256;
  P.ws_bytes = P.counters_bytes + (int64_t)P.pairs * P.max_contrib * sk::kRows * 16 * 4;
  return P;
}

}  // namespace sk_host

template <typename InT, int FMT, int SCALE, typename OutT, int NT, bool FUSED>
static int launch_sk(const GemvParams& p, int G, cudaStream_t st) {
  constexpr int KC = sk_host::kKC, STAGES = sk_host::kStages;
  auto kern = gemv_fp8_streamk_kernel<InT, FMT, SCALE, OutT, NT, FUSED, KC, STAGES>;
  const int smem = STAGES * sk::Cfg<KC>::kStageBytes + sk::kConsumers * sk::kRows * NT * 8 * 4;
  static unsigned attr_set = 0;  // per instantiation, one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned bit = 1u << (dev & 31);
  if (!(attr_set & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return CEK_ERR_LAUNCH;
    attr_set |= bit;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(sk::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

template <typename InT, typename OutT, bool FUSED>
static int sk_dispatch(const GemvParams& p, int G, int nt, int w_fmt, int scale_kind, cudaStream_t st) {
#define CEK_SK(F, S)                                                                         \
  if (w_fmt == F && scale_kind == S)                                                         \
    return nt == 1 ? launch_sk<InT, F, S, OutT, 1, FUSED>(p, G, st)                          \
                   : launch_sk<InT, F, S, OutT, 2, FUSED>(p, G, st);
  CEK_SK(CEK_E4M3, CEK_SCALE_PERN_F16)
  CEK_SK(CEK_E4M3, CEK_SCALE_PERN_F32)
  CEK_SK(CEK_E4M3, CEK_SCALE_PERT_F32)
  CEK_SK(CEK_E5M2, CEK_SCALE_PERN_F16)
  CEK_SK(CEK_E5M2, CEK_SCALE_PERN_F32)
  CEK_SK(CEK_E5M2, CEK_SCALE_PERT_F32)
#undef CEK_SK
  return CEK_ERR_INVALID_ARG;
}

int64_t gemv_streamk_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || M > 16 || N <= 0 || K <= 0) return 0;
  return sk_host::plan(M, N, K, sk_host::num_sms()).ws_bytes;
}

int gemv_streamk_launch(const GemvParams& base, int x_dtype, int y_dtype, int w_fmt, int scale_kind,
                        bool fused, void* workspace, int64_t ws_bytes, cudaStream_t st) {
  const sk_host::Plan P = sk_host::plan(base.M, base.N, base.K, sk_host::num_sms());
  if (ws_bytes < P.ws_bytes) return CEK_ERR_INVALID_ARG;
  GemvParams p = base;
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + P.counters_bytes);
  p.max_contrib = P.max_contrib;
  p.uk = P.uk;
  p.pairs = P.pairs;
  if (fused) {
    if (x_dtype != y_dtype) return CEK_ERR_INVALID_ARG;
    if (x_dtype == CEK_F16) return sk_dispatch<__half, __half, true>(p, P.G, P.nt, w_fmt, scale_kind, st);
    return sk_dispatch<__nv_bfloat16, __nv_bfloat16, true>(p, P.G, P.nt, w_fmt, scale_kind, st);
  }
  if (x_dtype == CEK_F16 && y_dtype == CEK_F16)
    return sk_dispatch<__half, __half, false>(p, P.G, P.nt, w_fmt, scale_kind, st);
  if (x_dtype == CEK_F16 && y_dtype == CEK_BF16)
    return sk_dispatch<__half, __nv_bfloat16, false>(p, P.G, P.nt, w_fmt, scale_kind, st);
  if (x_dtype == CEK_BF16 && y_dtype == CEK_F16)
    return sk_dispatch<__nv_bfloat16, __half, false>(p, P.G, P.nt, w_fmt, scale_kind, st);
  return sk_dispatch<__nv_bfloat16, __nv_bfloat16, false>(p, P.G, P.nt, w_fmt, scale_kind, st);
}

}  // namespace cek
