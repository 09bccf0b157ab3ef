// gemv_fp8_bulk.cu — the decode GEMV (M <= 16) as a bulk-copy stream.
//
//   y[m, n] = OutT( sum_k x[m, k] * deq(w[n, k]) * scale(n) )
//
// Same contract as the split-K kernel in gemv_fp8.cu (the reference's
// GEMV_fp8_pern_kernel / GEMV_fp8_pert_kernel, csrc/xpu/esimd_kernels/
// fp8_GEMV_v2.h:44-90, 322-368); this is the path for up to 16 tokens and
// K % 64 == 0.
//
// Why a second kernel.  With register-held weights every warp spends the
// FP8 conversion and MMA time of a batch before it reissues that batch's
// loads, so the bytes in flight per SM drop below what HBM needs, and each
// warp walks 16 rows 4 KB apart, which costs DRAM row locality.  Measured on
// gate_up (28672 x 4096, CUDA graph, cold L2): loads alone 18.9 us, the
// register kernel 31 us, this kernel 21-22 us.  The weight stream is
// decoupled from the math:
//  * Persistent grid, one CTA per SM (grid = min(SMs, N / 16)).  CTA c owns
//    the contiguous rows [N c / G, N (c + 1) / G): every CTA streams the same
//    byte count to within one row, with no cross-CTA reduction, because a
//    row's output needs only that row.
//  * Warp 0: producer.  A row block is 16 rows.  Consecutive rows are
//    contiguous in memory, so with whole rows per slab (K small enough) a
//    slab is one contiguous range, copied with 1-D cp.async.bulk in 8 KB
//    parts; for long rows K is cut into P pieces and a slab is 16 row
//    segments, one copy per lane.  Slabs land in a ring in shared memory
//    (completion by transaction-count mbarriers; no multicast).  x [M, K] is
//    copied once per CTA when it fits beside two slabs; otherwise (e.g.
//    M = 8, K = 14336) the consumers read it from L2 in batches of 8 chunks.
//  * Warps 1-8: consumers.  The 16 slab rows are the A operand of an
//    mma.sync m16n8k16, the tokens the 8 B columns (tokens >= M compute
//    values that are never stored); each consumer takes every 8th 64-k chunk
//    of a slab, converts its FP8 bytes exactly to f16x2 / bf16x2 and
//    accumulates in fp32 across the K pieces of the row block.  A stage is
//    handed back right after its last shared-memory read; the 8 partial sums
//    of a row block are reduced through shared memory in a fixed order
//    (deterministic results), scaled, converted and stored.
//  * K permutation: lane (g, t) reads 16 contiguous bytes of rows g and g+8
//    at k = 64c + 16t and the 16 matching activations of token g; word q
//    feeds MMA step q.  Any k bijection shared by both operands leaves the
//    sum unchanged.
//  * PDL: griddepcontrol.launch_dependents at CTA start; x is copied after
//    griddepcontrol.wait; with `early_weights` the first slabs are requested
//    before the wait.  The shared copy of x then lands behind those slabs,
//    so the consumers read x from L2 until it has arrived (measured: the
//    first MMA ~2.5 us earlier per launch).
//  * Every mbarrier wait is bounded.  A wait that gives up is counted
//    (cek_gemv_fp8_timeouts); the CTA stops waiting but keeps its barrier
//    sequence, so it always exits.
#include "gemv.cuh"
#include "mbarrier.cuh"

#include <algorithm>

namespace cek {
namespace bulk {

constexpr int kConsumers = 8;
constexpr int kAcc = 2;  // independent accumulators (shorter MMA dependency chains)
constexpr int kThreads = 32 * (1 + kConsumers);
constexpr int kSlabRows = 16;  // a row block: the m16 A operand of the MMA
constexpr int kMaxStages = 8;
constexpr uint32_t kPiece = 8192;  // bytes per bulk copy of a contiguous slab (16 / 32 KB: no faster)
constexpr int kSmemBudget = 216 * 1024;    // dynamic shared memory per CTA (static: ~8.3 KB)
constexpr uint32_t kWaitPolls = 1u << 22;
constexpr int kXBatch = 8;                 // chunks per batch when x is read from global memory
constexpr int kUnroll = 2;                 // chunk loop unroll when x is in shared memory
// Where the consumers read x from: shared memory (copied once per CTA), L2,
// or tensor memory (each consumer warp's chunks of x, stored once per CTA:
// used when x does not fit in shared memory beside two slabs).
constexpr int kXSmem = 0, kXL2 = 1, kXTmem = 2;
constexpr int kTmemCols = 512;             // all of TMEM: 256 columns per consumer warp
// Two CTAs per SM (CO = 1, the default for up to 8 tokens): half the shared
// memory (113 KB a CTA, static part included), half of TMEM and <= 96
// registers a thread, and a grid of two CTAs per SM, each streaming half of
// the SM's rows.  The SM keeps as many bytes in flight as one big CTA did,
// and when one CTA exits the next launch's CTA takes its place (prefetching
// its first slabs) while the other still drains, so consecutive launches
// overlap at their boundary.  Config-1 step (12 launches): 205.7 -> 179.9 us.
constexpr int kCoSmemPerCta = 113 * 1024;
__host__ __device__ constexpr int tmem_cols(int co) { return co ? kTmemCols / 2 : kTmemCols; }

__device__ unsigned long long g_timeouts;
#ifdef CEK_BULK_TRACE
__device__ unsigned long long g_trace[8192][8];
__device__ unsigned int g_trace_n;
CEK_DEVICE unsigned long long gtime() { unsigned long long t; asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)); return t; }
#define TRACE(slot, idx) do { if ((slot) < 8192) g_trace[(slot)][(idx)] = gtime(); } while (0)
#else
#define TRACE(slot, idx) do { } while (0)
#endif

// x_bytes: x staged in shared memory; ks: bytes of a row per slab (K / pieces);
// slab_bytes = 16 * ks.
// cl: CTAs per cluster splitting each row block along K (0 = no split).
struct Plan { int x_bytes, ks, pieces, pitch, slab_bytes, stages, smem, grid, xmode, nt, co, cl; };

// ---- K split over a thread-block cluster -------------------------------------
// For shapes with fewer 16-row blocks than SMs (a tensor-parallel shard of a
// short weight: 512 rows x 14336 at 8-way), the row blocks alone would leave
// most SMs idle.  Then a cluster of C CTAs shares one row block: CTA r of the
// cluster streams the K slice [r K / C, (r + 1) K / C) of its 16 rows (and
// the same slice of x), and the non-leader CTAs write their partial row sums
// into the leader's shared memory (distributed shared memory, st.shared::
// cluster) and arrive on the leader's mbarrier (release at cluster scope);
// the leader waits for them (bounded, acquire at cluster scope), adds the
// partial sums in rank order (deterministic) and runs the epilogue.  No
// global scratch.  Every CTA ends with a cluster barrier, so no CTA exits
// while another may still write into its shared memory.
CEK_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
CEK_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
CEK_DEVICE uint32_t map_leader(uint32_t saddr_local) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(saddr_local));
  return r;
}
CEK_DEVICE void st_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
CEK_DEVICE void arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
CEK_DEVICE bool wait_cluster(uint32_t bar, uint32_t parity, uint32_t polls) {
  for (uint32_t i = 0; i < polls; ++i) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    if (ok) return true;
  }
  return false;
}
constexpr int kMaxCluster = 8;

// Row blocks over the rows of one matrix, or of up to kMaxMats matrices
// sharing x (multi-GEMV, rows concatenated): a block is at most `bsz` rows
// (16; 8 gate/up row pairs for the gated GeLU output) and never straddles two
// matrices.
CEK_DEVICE int mat_rows(const GemvParams& p, int m) { return p.nmat ? p.mns[m] : p.N; }
CEK_DEVICE int total_rows(const GemvParams& p) {
  int t = 0;
  for (int m = 0; m < (p.nmat ? p.nmat : 1); ++m) t += mat_rows(p, m);
  return t;
}
struct BlockCursor {
  int m, mstart;  // current matrix and its first row in the concatenated numbering
  int row;        // next concatenated row
  int end;        // the CTA's end row
  int bsz;        // rows per block
  CEK_DEVICE void init(const GemvParams& p, int r0, int r1, int block_rows) {
    m = 0; mstart = 0; row = r0; end = r1; bsz = block_rows;
    while (m + 1 < (p.nmat ? p.nmat : 1) && row >= mstart + mat_rows(p, m)) mstart += mat_rows(p, m++);
  }
  // the next block: matrix, first row inside the matrix, row count
  CEK_DEVICE void next(const GemvParams& p, int& bm, int& brow, int& brows) {
    const int mend = mstart + mat_rows(p, m);
    const int stop = min(min(row + bsz, end), mend);
    bm = m; brow = row - mstart; brows = stop - row;
    row = stop;
    if (row == mend && m + 1 < (p.nmat ? p.nmat : 1)) { mstart = mend; ++m; }
  }
};
CEK_DEVICE int count_blocks(const GemvParams& p, int r0, int r1, int bsz) {
  int n = 0, ms = 0;
  for (int m = 0; m < (p.nmat ? p.nmat : 1); ++m) {
    const int me = ms + mat_rows(p, m);
    const int lo = max(r0, ms), hi = min(r1, me);
    if (hi > lo) n += (hi - lo + bsz - 1) / bsz;
    ms = me;
  }
  return n;
}

// NT: 8-token groups (the n8 columns of the MMA), 1 for M <= 8, 2 for M <= 16.
// NORM: the residual add + RMSNorm prologue (GemvParams::norm).
// CL: K split over a cluster of pl.cl CTAs (one 16-row block per cluster).
template <typename InT, int FMT, int SCALE, typename OutT, int XM, int NT, bool NORM, int CO = 0, bool CL = false>
__global__ void __launch_bounds__(kThreads, CO ? 2 : 1)
gemv_bulk_kernel(const GemvParams p, const Plan pl) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], xbar;
  __shared__ uint32_t tmem_base;
  __shared__ float red[2][kConsumers][kSlabRows][8 * NT];  // [row block parity][consumer][row][token]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.K, KS = pl.ks, P = pl.pieces;
  const int nrows = total_rows(p);
  // K split: this CTA's slice [koff, koff + KC) of every row and of x
  const int crank = CL ? (int)cluster_rank() : 0;
  const int KC = CL ? K / pl.cl : K, koff = crank * KC;
  const int r0 = CL ? (int)(blockIdx.x / pl.cl) * kSlabRows
                    : (int)((int64_t)nrows * blockIdx.x / gridDim.x);
  const int r1 = CL ? min(nrows, r0 + kSlabRows) : (int)((int64_t)nrows * (blockIdx.x + 1) / gridDim.x);
  __shared__ float cred[CL ? kMaxCluster : 1][CL ? kSlabRows : 1][CL ? 8 : 1];  // partial sums (leader)
  __shared__ __align__(8) uint64_t credbar;
  // gated GeLU output: a block is 8 gate rows (slab rows 0-7) and the
  // matching 8 up rows N + j (slab rows 8-15); rows count row pairs
  const int bsz = p.y_gelu ? kSlabRows / 2 : kSlabRows;
  const int nblocks = count_blocks(p, r0, r1, bsz);
  const int nslabs = nblocks * P;  // slab i = row block i / P, K piece i % P
  const int stages = pl.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar::init(mbar::saddr(&full[s]), 1);
      mbar::init(mbar::saddr(&empty[s]), kConsumers);
    }
    mbar::init(mbar::saddr(&xbar), 1);
    // the leader's reduction barrier: one arrival per epilogue thread of
    // every other CTA of the cluster
    if (CL) mbar::init(mbar::saddr(&credbar), (uint32_t)(pl.cl - 1) * kSlabRows * 8);
    mbar::fence_init();
  }
  __syncthreads();
  // the leader's barrier is initialised before any CTA of the cluster arrives
  if constexpr (CL) cluster_sync_all();
  if constexpr (!NORM) pdl_launch_dependents();
#ifdef CEK_BULK_TRACE
  __shared__ unsigned trace_slot;
  if (threadIdx.x == 0) {
    trace_slot = atomicAdd(&g_trace_n, 1u);
    if (trace_slot < 8192) { g_trace[trace_slot][0] = (unsigned long long)p.N * 1000000ull + p.M; g_trace[trace_slot][1] = blockIdx.x; }
    TRACE(trace_slot, 2);
  }
  __syncthreads();
  const unsigned tslot = trace_slot;
#else
  const unsigned tslot = 0;
#endif

  if (warp == 0) {
    // Producer warp.  A whole-row slab (P == 1) is one contiguous range,
    // copied by lane 0 in kPiece parts; a K piece of 16 rows is 16 row
    // segments, one copy per lane.
    const uint32_t ring = mbar::saddr(smem + pl.x_bytes);
    bool ok = true;
    BlockCursor cur;
    cur.init(p, r0, r1, bsz);
    int bm = 0, brow = 0, rows = 0;
    auto issue = [&](int i) {
      const int s = i % stages, pc = i % P;
      if (pc == 0) cur.next(p, bm, brow, rows);
      const uint8_t* wm = (p.nmat ? p.mws[bm] : p.w) + (size_t)brow * K + koff;
      const uint32_t dst = ring + (uint32_t)s * pl.slab_bytes;
      const uint32_t bar = mbar::saddr(&full[s]);
      if (lane == 0) mbar::arrive_expect_tx(bar, (p.y_gelu ? 2u : 1u) * (uint32_t)rows * (uint32_t)KS);
      __syncwarp();
      if (!CL && P == 1 && pl.pitch == KS) {
        if (lane == 0) {
          const uint32_t bytes = (uint32_t)rows * (uint32_t)K;
          for (uint32_t off = 0; off < bytes; off += kPiece)
            mbar::bulk_g2s(dst + off, wm + off, min(kPiece, bytes - off), bar);
          if (p.y_gelu) {
            const uint8_t* wu = wm + (size_t)p.N * K;
            for (uint32_t off = 0; off < bytes; off += kPiece)
              mbar::bulk_g2s(dst + 8u * pl.pitch + off, wu + off, min(kPiece, bytes - off), bar);
          }
        }
      } else if (!p.y_gelu) {
        if (lane < rows)
          mbar::bulk_g2s(dst + (uint32_t)lane * pl.pitch, wm + (size_t)lane * K + (size_t)pc * KS, (uint32_t)KS, bar);
      } else if (lane < 16 && (lane & 7) < rows) {
        const uint8_t* src = wm + (lane >= 8 ? (size_t)p.N * K : 0) + (size_t)(lane & 7) * K + (size_t)pc * KS;
        mbar::bulk_g2s(dst + (uint32_t)lane * pl.pitch, src, (uint32_t)KS, bar);
      }
    };
    const int pre = min(stages, nslabs);
    if (p.early_weights)
      for (int i = 0; i < pre; ++i) issue(i);
    pdl_wait();
    if (lane == 0) TRACE(tslot, 3);
    if (XM == kXSmem && lane == 0 && !NORM) {
      const uint32_t xb = (uint32_t)p.M * (uint32_t)K * 2u;
      const uint32_t bar = mbar::saddr(&xbar);
      const uint8_t* xs = static_cast<const uint8_t*>(p.x);
      if constexpr (CL) {
        // this CTA's K slice of every token's row, packed with row length KC
        const uint32_t rb = (uint32_t)KC * 2u;
        mbar::arrive_expect_tx(bar, (uint32_t)p.M * rb);
        for (int m = 0; m < p.M; ++m)
          for (uint32_t off = 0; off < rb; off += kPiece)
            mbar::bulk_g2s(mbar::saddr(smem) + (uint32_t)m * rb + off, xs + ((size_t)m * K + koff) * 2u + off,
                           min(kPiece, rb - off), bar);
      } else {
        mbar::arrive_expect_tx(bar, xb);
        for (uint32_t off = 0; off < xb; off += kPiece)
          mbar::bulk_g2s(mbar::saddr(smem) + off, xs + off, min(kPiece, xb - off), bar);
      }
    }
    if (!p.early_weights)
      for (int i = 0; i < pre; ++i) issue(i);
    int issued = pre;
    for (int i = pre; i < nslabs && ok; ++i) {
      // stage i % stages is free once the consumers released use (i / stages) - 1
      if (lane == 0) ok = mbar::wait(mbar::saddr(&empty[i % stages]), ((i / stages) + 1) & 1, kWaitPolls);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicAdd(&g_timeouts, 1ull);
        break;  // the consumers' waits run out too
      }
      issue(i);
      issued = i + 1;
    }
    if (lane == 0) TRACE(tslot, 4);
    // The CTA's shared memory must outlive every copy into it, also when a
    // consumer gave up waiting and exits early: wait (bounded) until the
    // last `stages` slabs issued have landed.  Slab j's phase of stage
    // j % stages cannot be overtaken, because nothing later was issued there.
    if (lane == 0)
      for (int j = max(0, issued - stages); j < issued; ++j)
        if (!mbar::wait(mbar::saddr(&full[j % stages]), (j / stages) & 1, kWaitPolls)) {
          atomicAdd(&g_timeouts, 1ull);
          break;
        }
    if constexpr (CL) cluster_sync_all();
    return;
  }

  // ---- consumers ----
  const int cw = warp - 1, g = lane >> 2, t = lane & 3;
  const int ctid = threadIdx.x - 32;
  // Lane (g, t) carries tokens g + 8u of the NT groups.  Tokens >= M read
  // token 0's activations: their output columns are never stored.
  uint32_t xrow[NT];
  const InT* xglob[NT];
#pragma unroll
  for (int u = 0; u < NT; ++u) {
    const int xtok = g + 8 * u < p.M ? g + 8 * u : 0;
    xrow[u] = mbar::saddr(smem) + (uint32_t)xtok * KC * 2u + 32u * t;
    xglob[u] = reinterpret_cast<const InT*>(p.x) + (size_t)xtok * K + koff + 16 * t;
  }
  const int nchunks = KS / 64;
  bool dead = false;
  // x may be read from global memory (L2) only after the previous kernel
  // has completed; the shared-memory copy of x arrives behind the weight
  // slabs requested early, so until it lands the slabs use the global path.
  pdl_wait();
  bool x_smem = false;
  // Norm prologue, pass 1 (all consumer threads, token by token): the sum of
  // squares of the unrounded h + r, reduced over the CTA into the inverse
  // RMS; with x in shared memory the rounded residual io(h + r) is stored
  // there on the way.
  __shared__ float ninv[NORM ? 16 : 1];
  __shared__ float nred[NORM ? kConsumers : 1][NORM ? 16 : 1];
  if constexpr (NORM) {
    const int nvec = K >> 3;
#pragma unroll 2
    for (int m = 0; m < p.M; ++m) {
      const uint4* hv = reinterpret_cast<const uint4*>(static_cast<const InT*>(p.x) + (size_t)m * K);
      const uint4* rv = reinterpret_cast<const uint4*>(static_cast<const InT*>(p.residual) + (size_t)m * K);
      float ss = 0.f;
#pragma unroll 4
      for (int v = ctid; v < nvec; v += kConsumers * 32) {
        const uint4 h = ldg_nc(hv + v), r = ldg_nc(rv + v);
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, rw[4] = {r.x, r.y, r.z, r.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 hf = unpack2<InT>(hw[q]), rf = unpack2<InT>(rw[q]);
          const float a = hf.x + rf.x, b = hf.y + rf.y;
          ss += a * a + b * b;
          o[q] = pack2<InT>(a, b);
        }
        if (XM == kXSmem) reinterpret_cast<uint4*>(smem + (size_t)m * K * 2)[v] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      ss = warp_sum(ss);
      if (lane == 0) nred[cw][m] = ss;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    if (ctid < p.M) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < kConsumers; ++q) t += nred[q][ctid];
      ninv[ctid] = rsqrtf(t / (float)K + p.eps);
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
  }
  // pass 2 helper (x in tensor memory): the 16 normalised activations of
  // token tok at k .. k + 15, io(f32(io(h + r)) * inv_rms * gamma), the
  // rounding points of the two-kernel path
  auto norm16 = [&](int tok, int k, uint4& a, uint4& b) {
    const InT* hp = static_cast<const InT*>(p.x) + (size_t)tok * K + k;
    const InT* rp = static_cast<const InT*>(p.residual) + (size_t)tok * K + k;
    const InT* gp = static_cast<const InT*>(p.gamma) + k;
    const float inv = ninv[tok];
    uint32_t o[8];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint4 h = ldg_nc(hp + 8 * half), r = ldg_nc(rp + 8 * half), gm = ldg_nc(gp + 8 * half);
      const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, rw[4] = {r.x, r.y, r.z, r.w}, gw[4] = {gm.x, gm.y, gm.z, gm.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 hf = unpack2<InT>(hw[q]), rf = unpack2<InT>(rw[q]), gf = unpack2<InT>(gw[q]);
        const float2 res = unpack2<InT>(pack2<InT>(hf.x + rf.x, hf.y + rf.y));
        o[4 * half + q] = pack2<InT>(res.x * inv * gf.x, res.y * inv * gf.y);
      }
    }
    a = make_uint4(o[0], o[1], o[2], o[3]);
    b = make_uint4(o[4], o[5], o[6], o[7]);
  };
  if (XM == kXSmem && NORM) {
    // pass 2 in place: x[m][k] = io(x[m][k] * inv_rms[m] * gamma[k])
    const int nvec = K >> 3;
    for (int e = ctid; e < p.M * nvec; e += kConsumers * 32) {
      const int m = e / nvec, v = e - m * nvec;
      uint4* xp = reinterpret_cast<uint4*>(smem + (size_t)m * K * 2) + v;
      const uint4 x4 = *xp, gm = ldg_nc(static_cast<const InT*>(p.gamma) + 8 * v);
      const uint32_t xw[4] = {x4.x, x4.y, x4.z, x4.w}, gw[4] = {gm.x, gm.y, gm.z, gm.w};
      const float inv = ninv[m];
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 xf = unpack2<InT>(xw[q]), gf = unpack2<InT>(gw[q]);
        o[q] = pack2<InT>(xf.x * inv * gf.x, xf.y * inv * gf.y);
      }
      *xp = make_uint4(o[0], o[1], o[2], o[3]);
    }
    x_smem = true;  // visible to all consumers after the barrier below
  }
  // tensor-memory copy of x: warp cw owns global chunks cw, cw + 8, ...; its
  // chunk j sits in columns [8 NT j, 8 NT (j + 1)) of its half of its lane
  // quadrant (warps cw and cw + 4 share the quadrant of warp index % 4),
  // lane (g, t) holding, per token group u, token g + 8u's 16 activations at
  // k = 64 chunk + 16 t in columns 8 NT j + 8u ..
  uint32_t xt = 0;
  if constexpr (XM == kXTmem) {
    if (cw == 0) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                   ::"r"(mbar::saddr(&tmem_base)), "r"(tmem_cols(CO)) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    xt = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (cw >= 4 ? tmem_cols(CO) / 2 : 0);
    if constexpr (!NORM) {
      for (int j = 0; cw + j * kConsumers < K / 64; ++j) {
#pragma unroll
        for (int u = 0; u < NT; ++u) {
          const InT* xq = xglob[u] + 64 * (cw + j * kConsumers);
          const uint4 a = ldg_nc(xq), b = ldg_nc(xq + 8);
          asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                       ::"r"(xt + 8u * (NT * j + u)), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y),
                         "r"(b.z), "r"(b.w) : "memory");
        }
      }
    } else {
      // two chunks per batch: all their loads issue before the first store
      const int nj = (K / 64 - cw + kConsumers - 1) / kConsumers;
      for (int j0 = 0; j0 < nj; j0 += 2) {
        uint4 a[2][NT], b[2][NT];
#pragma unroll
        for (int v = 0; v < 2; ++v)
#pragma unroll
          for (int u = 0; u < NT; ++u)
            norm16(g + 8 * u < p.M ? g + 8 * u : 0, 64 * (cw + min(j0 + v, nj - 1) * kConsumers) + 16 * t, a[v][u],
                   b[v][u]);
#pragma unroll
        for (int v = 0; v < 2; ++v)
#pragma unroll
          for (int u = 0; u < NT; ++u)
            if (j0 + v < nj)
              asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                           ::"r"(xt + 8u * (NT * (j0 + v) + u)), "r"(a[v][u].x), "r"(a[v][u].y), "r"(a[v][u].z),
                             "r"(a[v][u].w), "r"(b[v][u].x), "r"(b[v][u].y), "r"(b[v][u].z), "r"(b[v][u].w)
                           : "memory");
      }
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  }
  // the residual has been read for the last time: a kernel launched behind
  // this one may now update it in place
  if constexpr (NORM) {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    pdl_launch_dependents();
  }
  if (cw == 0 && lane == 0) TRACE(tslot, 5);

  // one 64-k chunk: rows g, g+8 (16 bytes each) against the 16 activations
  // of each token group (xa[u], xb[u]); the FP8 conversion is done once
  auto chunk_mma = [&](float (&ac)[NT][kAcc][4], const uint4& wa, const uint4& wb, const uint4 (&xa)[NT],
                       const uint4 (&xb)[NT]) {
    const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w}, rb4[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t a[4] = {cvt_pair<InT, FMT, 0>(ra[q]), cvt_pair<InT, FMT, 0>(rb4[q]),
                             cvt_pair<InT, FMT, 1>(ra[q]), cvt_pair<InT, FMT, 1>(rb4[q])};
#pragma unroll
      for (int u = 0; u < NT; ++u) {
        const uint32_t b0 = (q < 2) ? ((q == 0) ? xa[u].x : xa[u].z) : ((q == 2) ? xb[u].x : xb[u].z);
        const uint32_t b1 = (q < 2) ? ((q == 0) ? xa[u].y : xa[u].w) : ((q == 2) ? xb[u].y : xb[u].w);
        mma16816<InT>(ac[u][q % kAcc], a, b0, b1);
      }
    }
  };

  float acc[NT][kAcc][4];
  float out_scale = 0.f, out_scale_up = 0.f;
  int out_row = 0;  // row inside the block's matrix of this thread's output
  bool out_ok = false;
  int bm = 0, brow = 0, brows = 0;
  BlockCursor cur;
  cur.init(p, r0, r1, bsz);
  for (int i = 0; i < nslabs; ++i) {
    const int s = i % stages, rb = i / P, pc = i - rb * P;
    if (pc == 0) {
      // new row block: clear the sums; the epilogue thread fetches its scale
      // now, so the load's latency hides behind the block's math
      cur.next(p, bm, brow, brows);
#pragma unroll
      for (int u = 0; u < NT; ++u)
#pragma unroll
        for (int a = 0; a < kAcc; ++a) acc[u][a][0] = acc[u][a][1] = acc[u][a][2] = acc[u][a][3] = 0.f;
      out_row = brow + (ctid % bsz);
      out_ok = ctid < bsz * 8 * NT && (ctid % bsz) < brows;
      out_scale = out_ok ? load_scale<SCALE>(p.nmat ? p.mscales[bm] : p.scale, out_row) : 0.f;
      if (p.y_gelu) out_scale_up = out_ok ? load_scale<SCALE>(p.scale, p.N + out_row) : 0.f;
    }
    if (!dead && !mbar::wait(mbar::saddr(&full[s]), (i / stages) & 1, kWaitPolls)) {
      dead = true;
      if (lane == 0) atomicAdd(&g_timeouts, 1ull);
    }
    dead = __any_sync(0xffffffffu, dead);  // warp-uniform: the tensor-memory loads are warp-collective
    if (i == 0 && cw == 0 && lane == 0) TRACE(tslot, 7);
    const uint32_t wrow = mbar::saddr(smem + pl.x_bytes) + (uint32_t)s * pl.slab_bytes + (uint32_t)g * pl.pitch + 16u * t;
    const uint32_t wrow8 = wrow + 8u * pl.pitch;
    if (XM == kXSmem && !x_smem) x_smem = __shfl_sync(0xffffffffu, lane == 0 ? mbar::try_wait(mbar::saddr(&xbar), 0) : false, 0);
    if (!dead) {
      if constexpr (XM == kXTmem) {
        // chunk c of piece pc is global chunk pc * nchunks + c, the warp's
        // chunk (that / 8), columns 8 NT (that / 8) + 8u
        const uint32_t xcol = xt + 8u * NT * (uint32_t)((pc * nchunks + cw) / kConsumers);
        for (int c = cw; c < nchunks; c += 2 * kConsumers) {
          // two chunks per tensor-memory wait
          const bool two = c + kConsumers < nchunks;
          const uint32_t col = xcol + 8u * NT * (uint32_t)((c - cw) / kConsumers);
          uint4 xa[2][NT], xb[2][NT];
#pragma unroll
          for (int v = 0; v < 2; ++v)
#pragma unroll
            for (int u = 0; u < NT; ++u)
              if (v == 0 || two)
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(xa[v][u].x), "=r"(xa[v][u].y), "=r"(xa[v][u].z), "=r"(xa[v][u].w),
                               "=r"(xb[v][u].x), "=r"(xb[v][u].y), "=r"(xb[v][u].z), "=r"(xb[v][u].w)
                             : "r"(col + 8u * (NT * v + u)));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          chunk_mma(acc, mbar::lds16(wrow + 64u * c), mbar::lds16(wrow8 + 64u * c), xa[0], xb[0]);
          if (two)
            chunk_mma(acc, mbar::lds16(wrow + 64u * (c + kConsumers)), mbar::lds16(wrow8 + 64u * (c + kConsumers)),
                      xa[1], xb[1]);
        }
      } else if (x_smem) {
#pragma unroll (CO ? 1 : kUnroll)
        for (int c = cw; c < nchunks; c += kConsumers) {
          uint4 xa[NT], xb[NT];
#pragma unroll
          for (int u = 0; u < NT; ++u) {
            const uint32_t xq = xrow[u] + (uint32_t)pc * KS * 2u + 128u * c;
            xa[u] = mbar::lds16(xq);
            xb[u] = mbar::lds16(xq + 16u);
          }
          chunk_mma(acc, mbar::lds16(wrow + 64u * c), mbar::lds16(wrow8 + 64u * c), xa, xb);
        }
      } else {
        // x from L2: a batch of kXBatch / NT chunks issues all its activation
        // loads before the first MMA
        constexpr int XB = kXBatch / NT / (CO ? 2 : 1);
        for (int c0 = cw; c0 < nchunks; c0 += XB * kConsumers) {
          uint4 xa[XB][NT], xb[XB][NT];
#pragma unroll
          for (int v = 0; v < XB; ++v) {
            const int c = min(c0 + v * kConsumers, nchunks - 1);
#pragma unroll
            for (int u = 0; u < NT; ++u) {
              const InT* xq = xglob[u] + (size_t)pc * KS + 64 * c;
              xa[v][u] = ldg_nc(xq);
              xb[v][u] = ldg_nc(xq + 8);
            }
          }
#pragma unroll
          for (int v = 0; v < XB; ++v) {
            const int c = c0 + v * kConsumers;
            if (c < nchunks) chunk_mma(acc, mbar::lds16(wrow + 64u * c), mbar::lds16(wrow8 + 64u * c), xa[v], xb[v]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar::arrive(mbar::saddr(&empty[s]));
    if (pc != P - 1) continue;
    float (&rd)[kConsumers][kSlabRows][8 * NT] = red[rb & 1];
#pragma unroll
    for (int u = 0; u < NT; ++u) {
      float v4[4] = {acc[u][0][0], acc[u][0][1], acc[u][0][2], acc[u][0][3]};
#pragma unroll
      for (int a = 1; a < kAcc; ++a)
#pragma unroll
        for (int e = 0; e < 4; ++e) v4[e] += acc[u][a][e];
      // v4[0..1]: block row g, tokens 8u + 2t, 8u + 2t + 1; v4[2..3]: row g + 8
      rd[cw][g][8 * u + 2 * t] = v4[0];
      rd[cw][g][8 * u + 2 * t + 1] = v4[1];
      rd[cw][g + 8][8 * u + 2 * t] = v4[2];
      rd[cw][g + 8][8 * u + 2 * t + 1] = v4[3];
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    if (ctid < bsz * 8 * NT) {
      const int tok = ctid / bsz, row = ctid % bsz;
      if constexpr (CL) {
        // K split: the other CTAs hand their partial sums to the leader
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kConsumers; ++q) v += rd[q][row][tok];
        if (crank != 0) {
          st_cluster_f32(map_leader(mbar::saddr(&cred[crank][row][tok])), v);
          arrive_remote(map_leader(mbar::saddr(&credbar)));
          continue;
        }
        if (!wait_cluster(mbar::saddr(&credbar), 0, kWaitPolls)) atomicAdd(&g_timeouts, 1ull);
        for (int r = 1; r < pl.cl; ++r) v += cred[r][row][tok];
        if (tok < p.M && out_ok)
          store_out<OutT>(p, reinterpret_cast<OutT*>(p.y), p.N, tok, out_row, from_f32<OutT>(v * out_scale));
        continue;
      }
      if (tok < p.M && out_ok) {
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kConsumers; ++q) v += rd[q][row][tok];
        OutT o = from_f32<OutT>(v * out_scale);
        if (p.y_gelu) {
          // the up row of the pair sits 8 slab rows below the gate row; each
          // is rounded to the output type first, as the unfused GEMV stores
          // them, then io(gelu_tanh(gate) * up)
          float u = 0.f;
#pragma unroll
          for (int q = 0; q < kConsumers; ++q) u += rd[q][row + 8][tok];
          o = gelu_mul1<OutT>(o, from_f32<OutT>(u * out_scale_up));
        }
        store_out<OutT>(p, reinterpret_cast<OutT*>(p.nmat ? p.mys[bm] : p.y), p.nmat ? p.mns[bm] : p.N, tok,
                        out_row, o);
      }
    }
  }
  if constexpr (XM == kXTmem) {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory");
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (cw == 0)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols(CO)) : "memory");
  }
  // the CTA's shared memory must outlive the x copy into it
  if (XM == kXSmem && !x_smem && cw == 0 && !mbar::wait(mbar::saddr(&xbar), 0, kWaitPolls) && lane == 0)
    atomicAdd(&g_timeouts, 1ull);
  if (cw == 0 && lane == 0) TRACE(tslot, 6);
  // no CTA of the cluster leaves while the leader's shared memory may still
  // receive partial sums
  if constexpr (CL) cluster_sync_all();
}

// Shared-memory plan for M tokens and K; stages == 0 means "not applicable".
// K is cut into the fewest pieces (each a multiple of 64 bytes, and at least
// kMinRowCopy bytes when cut: smaller copies cost more than they stream)
// that leave room for x and `want` slabs.  When x [M, K] itself does not fit
// beside two slabs it is read from global memory (L2) instead.
constexpr int kMinRowCopy = 3072;
constexpr int kRowPad = 0;  // shared-memory row padding (16 measured no faster)

static bool try_plan(Plan& pl, int64_t x_bytes, int64_t K, int want, int64_t budget,
                     int64_t min_copy = kMinRowCopy) {
  const int64_t room = budget - x_bytes;
  if (room <= 0) return false;
  for (int64_t P = 1; P <= 16; ++P) {
    if (K % (64 * P) != 0) continue;
    const int64_t ks = K / P;
    if (P > 1 && ks < min_copy) break;
    const int64_t pitch = ks + kRowPad;
    const int64_t st = room / (kSlabRows * pitch);
    if (st >= want) {
      pl.x_bytes = (int)x_bytes;
      pl.pieces = (int)P;
      pl.ks = (int)ks;
      pl.pitch = (int)pitch;
      pl.slab_bytes = (int)(kSlabRows * pitch);
      pl.stages = (int)std::min<int64_t>(st, kMaxStages);
      return true;
    }
  }
  return false;
}

Plan plan(int64_t M, int64_t N, int64_t K, int co = 0, int gridx = 1, int64_t extra_static = 0,
          int64_t min_copy = 0) {
  Plan pl = {};
  if (M < 1 || M > 16 || K % 64 != 0 || K <= 0 || N <= 0 || K > (1 << 20)) return pl;
  const int nt = M <= 8 ? 1 : 2;
  if (co && nt != 1) return pl;
  // the static reduction array grows with the token groups (8 KB each)
  const int64_t budget = (co ? kCoSmemPerCta - 9 * 1024 : kSmemBudget - (nt - 1) * 8 * 1024) - extra_static;
  // two CTAs per SM: row pieces of at least 2 KB (16 copies of 1 KB per slab
  // measured 1.4-2x slower), and no two-slab plan (x from L2 instead)
  const int64_t mc = min_copy > 0 ? min_copy : co ? 2048 : kMinRowCopy;
  const int64_t xb = ((M * K * 2) + 127) / 128 * 128;
  // x in shared memory with three slabs; else x in tensor memory (when its
  // layout fits) with three slabs; else x in shared memory with two; else x
  // from L2.  Tensor memory holds 8 columns (one 64-k chunk of 16
  // activations per lane) per chunk and token group a warp owns: NT K / 64
  // columns per warp, 256 available, and chunk ownership (every 8th chunk)
  // must not change across K pieces.
  auto tmem_fits = [&](const Plan& q) {
    return K % 512 == 0 && nt * K / 64 <= tmem_cols(co) / 2 && (q.ks / 64) % kConsumers == 0;
  };
  Plan t = {};
  if (try_plan(pl, xb, K, 3, budget, mc)) {
    pl.xmode = kXSmem;
  } else if (try_plan(t, 0, K, 3, budget, mc) && tmem_fits(t)) {
    pl = t;
    pl.xmode = kXTmem;
  } else if (!co && try_plan(pl, xb, K, 2, budget, mc)) {
    pl.xmode = kXSmem;
  } else if (try_plan(pl, 0, K, 3, budget, mc)) {
    pl.xmode = kXL2;
  } else {
    return Plan{};
  }
  pl.nt = nt;
  pl.smem = pl.x_bytes + pl.stages * pl.slab_bytes;
  const int sms = cek_host::sm_count();
  pl.co = co;
  pl.grid = (int)std::min<int64_t>((int64_t)sms * (co ? gridx : 1), (N + kSlabRows - 1) / kSlabRows);
  return pl;
}

template <typename InT, int FMT, int SCALE, typename OutT, int XM, int NT, bool NORM = false, int CO = 0,
          bool CL = false>
int launch(const GemvParams& p, const Plan& pl, cudaStream_t st) {
  auto kern = gemv_bulk_kernel<InT, FMT, SCALE, OutT, XM, NT, NORM, CO, CL>;
  static cek_host::DeviceSlots configured_smem;
  // beside the static reduction array
  constexpr int kMaxDyn = CO ? kCoSmemPerCta - 9 * 1024 : kSmemBudget - (NT - 1) * 8 * 1024;
  if (!cek_host::ensure_smem_attr(configured_smem, kern, kMaxDyn)) return CEK_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (CL) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)pl.cl;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, p, pl) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

template <typename InT, int F, int S, typename OutT, int NT>
int launch_x(const GemvParams& p, const Plan& pl, cudaStream_t st) {
  // the norm prologue (e4m3 weights only) keeps x in shared or tensor memory
  if constexpr (F == CEK_E4M3)
    if (p.norm) {
      if constexpr (NT == 1)
        if (pl.co) return launch<InT, F, S, OutT, kXSmem, NT, true, 1>(p, pl, st);
      return launch<InT, F, S, OutT, kXSmem, NT, true>(p, pl, st);
    }
  if constexpr (F == CEK_E4M3 && NT == 1)
    if (pl.cl > 1)
      return pl.xmode == kXSmem ? launch<InT, F, S, OutT, kXSmem, NT, false, 1, true>(p, pl, st)
                                : launch<InT, F, S, OutT, kXL2, NT, false, 1, true>(p, pl, st);
  if constexpr (F == CEK_E4M3 && NT == 1)
    if (pl.co)
      return pl.xmode == kXSmem   ? launch<InT, F, S, OutT, kXSmem, NT, false, 1>(p, pl, st)
             : pl.xmode == kXTmem ? launch<InT, F, S, OutT, kXTmem, NT, false, 1>(p, pl, st)
                                  : launch<InT, F, S, OutT, kXL2, NT, false, 1>(p, pl, st);
  return pl.xmode == kXSmem   ? launch<InT, F, S, OutT, kXSmem, NT>(p, pl, st)
         : pl.xmode == kXTmem ? launch<InT, F, S, OutT, kXTmem, NT>(p, pl, st)
                              : launch<InT, F, S, OutT, kXL2, NT>(p, pl, st);
}

template <typename InT, typename OutT>
int dispatch(const GemvParams& p, const Plan& pl, int w_fmt, int scale_kind, cudaStream_t st) {
#define CEK_CASE(F, S) \
  if (w_fmt == F && scale_kind == S)                                    \
    return pl.nt == 1 ? launch_x<InT, F, S, OutT, 1>(p, pl, st) : launch_x<InT, F, S, OutT, 2>(p, pl, st);
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERN_F16)
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERN_F32)
  CEK_CASE(CEK_E4M3, CEK_SCALE_PERT_F32)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERN_F16)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERN_F32)
  CEK_CASE(CEK_E5M2, CEK_SCALE_PERT_F32)
#undef CEK_CASE
  return CEK_ERR_INVALID_ARG;
}

}  // namespace bulk

// The bulk path for a plain GEMV call, or CEK_ERR_UNSUPPORTED when the call
// does not fit it (more than 8 tokens or K % 64 != 0; the gated GeLU output
// also needs a single matrix without the all-reduce push).  x and w must be
// 16-byte aligned.
// K-split clusters: only for long rows (K >= kMinClusterK) and clusters of at
// least kMinCluster CTAs, in slices (and row pieces) of at least
// kMinClusterSlice bytes; kClusterStatic is the static shared memory the split
// adds (the leader's partial-sum array).  Measured (CUDA graph of calls over
// cold weights, M = 1 / 2 / 4 / 8; without -> with the split):
//   512 x 14336 (8 CTAs a cluster):  7.3 / 8.5 / 8.8 / 9.2 -> 6.5 / 6.8 / 6.9 / 6.7 us
//   1024 x 14336 (4):                7.6 / 8.8 / 9.1 / 9.4 -> 7.1 / 7.3 / 7.7 / 7.9 us
// and slower where the clusters are pairs or the rows shorter:
//   2048 x 14336 (2): 8.8 -> 9.1 us at M = 1; 1280 x 8192 (2): 5.9 -> 6.9 us;
//   640 x 8192 (4): 5.4 -> 5.4-5.8 us; 768 x 4096 (4, 1 KB slices): 3.9 -> 5.0 us.
constexpr int64_t kMinClusterK = 12288;
constexpr int kMinCluster = 4;
constexpr int64_t kMinClusterSlice = 1024;
constexpr int64_t kClusterStatic = 4 * 1024 + 64;

int gemv_bulk_launch(const GemvParams& p, int x_dtype, int y_dtype, int w_fmt, int scale_kind, cudaStream_t st) {
  static const bool disabled = [] {
    const char* v = std::getenv("CEK_GEMV_BULK");
    return v && v[0] == '0';
  }();
  if (disabled) return CEK_ERR_UNSUPPORTED;
  // Two CTAs per SM for up to 8 tokens (e4m3), unless CEK_BULK_CO=0;
  // CEK_BULK_GRIDX=1 gives one CTA per SM per launch (for measurement).
  static const int co_mode = [] {
    const char* v = std::getenv("CEK_BULK_CO");
    return v ? std::atoi(v) : 1;
  }();
  static const int gridx = [] {
    const char* v = std::getenv("CEK_BULK_GRIDX");
    const int g = v ? std::atoi(v) : 2;
    return g >= 1 && g <= 4 ? g : 2;
  }();
  bulk::Plan pl = {};
  // Fewer 16-row blocks than SMs (a short shard) and long rows: split every
  // row block along K over a cluster of C CTAs (the largest C in [4, 8] with
  // K / C a multiple of 64 of at least kMinClusterSlice bytes and at most two
  // CTAs per SM in all), two CTAs per SM.  CEK_BULK_CLUSTER=0 turns it off.
  static const int cluster_mode = [] {
    const char* v = std::getenv("CEK_BULK_CLUSTER");
    return v ? std::atoi(v) : 1;
  }();
  const int64_t nrows0 = p.y_gelu ? 2 * (int64_t)p.N : p.N;
  const int64_t nblk = (nrows0 + 15) / 16;
  const int sms0 = cek_host::sm_count();
  if (cluster_mode && w_fmt == CEK_E4M3 && !p.norm && !p.y_gelu && !p.nmat && p.M <= 8 && nblk < sms0 &&
      p.K >= kMinClusterK && x_dtype == y_dtype) {
    for (int c = bulk::kMaxCluster; c >= kMinCluster; --c) {
      if (p.K % (64 * c) != 0 || p.K / c < kMinClusterSlice || nblk * c > 2 * (int64_t)sms0) continue;
      // one row block per CTA: K pieces down to kMinClusterSlice bytes
      bulk::Plan q = bulk::plan(p.M, nrows0, p.K / c, 1, 2, kClusterStatic, kMinClusterSlice);
      if (q.stages == 0 || (q.xmode != bulk::kXSmem && q.xmode != bulk::kXL2)) continue;
      q.cl = c;
      q.grid = (int)(nblk * c);
      return x_dtype == CEK_F16 ? bulk::dispatch<__half, __half>(p, q, w_fmt, scale_kind, st)
                                : bulk::dispatch<__nv_bfloat16, __nv_bfloat16>(p, q, w_fmt, scale_kind, st);
    }
  }
  // ... when there are at least as many 16-row blocks as SMs: with fewer,
  // the grid is not two CTAs per SM anyway and the halved ring only costs
  // (e.g. one rank's down shard at 4- and 8-way tensor parallelism, 512 or
  // 1024 rows: 9.5 against 6.1 us)
  const int64_t nrows = p.y_gelu ? 2 * (int64_t)p.N : p.N;
  if (co_mode == 1 && w_fmt == CEK_E4M3 && (nrows + 15) / 16 >= cek_host::sm_count())
    pl = bulk::plan(p.M, nrows, p.K, 1, gridx);
  // the norm prologue needs x in shared memory: fall back to one CTA per SM
  if (p.norm && pl.stages && pl.xmode != bulk::kXSmem) pl = bulk::Plan{};
  if (pl.stages == 0) pl = bulk::plan(p.M, p.y_gelu ? 2 * (int64_t)p.N : p.N, p.K);
  if (pl.stages == 0 || (p.y_gelu && (p.nmat || p.ar_world))) return CEK_ERR_UNSUPPORTED;
  // the norm prologue needs x on chip and a single plain or gated matrix
  // The norm prologue runs where x fits in shared memory beside the ring (one
  // pass over h + r stores the residual there).  With x in tensor memory
  // (M >= 4 at K = 4096) it measured slower than the two-kernel path, which
  // the caller then takes.
  if (p.norm && (pl.xmode != bulk::kXSmem || p.nmat || p.ar_world || w_fmt != CEK_E4M3)) return CEK_ERR_UNSUPPORTED;
  // two token groups with x from L2 measured slower than the split-K kernel
  // (down 4096 x 14336 at M = 16: 24.3 against 22.5 us)
  if (pl.nt == 2 && pl.xmode == bulk::kXL2 && !p.y_gelu) return CEK_ERR_UNSUPPORTED;
  // mixed activation / output types stay on the split-K kernel
  if (x_dtype != y_dtype) return CEK_ERR_UNSUPPORTED;
  if (x_dtype == CEK_F16) return bulk::dispatch<__half, __half>(p, pl, w_fmt, scale_kind, st);
  return bulk::dispatch<__nv_bfloat16, __nv_bfloat16>(p, pl, w_fmt, scale_kind, st);
}

}  // namespace cek

#ifdef CEK_BULK_TRACE
extern "C" int cek_bulk_trace_read(unsigned long long* host, unsigned* n) {
  cudaMemcpyFromSymbol(n, cek::bulk::g_trace_n, 4);
  cudaMemcpyFromSymbol(host, cek::bulk::g_trace, sizeof(unsigned long long) * 8192 * 8);
  unsigned z = 0;
  cudaMemcpyToSymbol(cek::bulk::g_trace_n, &z, 4);
  return 0;
}
#endif

extern "C" int cek_gemv_fp8_timeouts(uint64_t* count) {
  if (!count) return CEK_ERR_INVALID_ARG;
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, cek::bulk::g_timeouts, sizeof(v)) != cudaSuccess) return CEK_ERR_LAUNCH;
  *count = v;
  return CEK_OK;
}
