// gemm_fp8_tcgen05.cu — prefill FP8 x FP8 GEMM on the 5th-generation tensor
// cores (tcgen05), per-token x per-channel scales in the epilogue.
//
//   y[m, n] = OutT( (sum_k deq(aq[m, k]) * deq(bq[n, k])) * a_scale[m] * b_scale[n] )
//
// This replaces the reference's prefill route (GEMM_fp8_pert_dispatch sends
// M > 64 to a scalar weight-stationary kernel, csrc/xpu/esimd_kernels/
// fp8_GEMM_pert.h:165-210, 4043-4048).
//
// Layout: persistent kernel, one CTA per SM, 6 warps.
//  * warp 0 (one lane): TMA producer.  128x128-byte A boxes and 256x128-byte
//    B boxes (128-byte swizzle) into a 4-stage shared-memory ring, completion
//    by transaction-count mbarriers.  No multicast.
//  * warp 1: allocates 512 TMEM columns (two 128x256 fp32 accumulators) and
//    one lane issues tcgen05.mma kind::f8f6f4 (M=128, N=256, K=32 per
//    instruction, 4 per stage); tcgen05.commit releases each smem stage and
//    signals each finished accumulator.
//  * warps 2-5: epilogue.  tcgen05.ld 32 columns at a time from their TMEM
//    lane quadrant, scale, convert, store; then hand the accumulator back so
//    the MMA warp can start the tile after next while this one drains.
//  Tiles are 128 (M) x 256 (N); tile t covers m-block t % num_m and n-block
//  t / num_m, so the CTAs in flight share B blocks through L2.
//  Every mbarrier wait is bounded: on timeout the CTA records it in a device
//  counter (cek_gemm_fp8_timeouts), stops, waits (bounded) for its own copies
//  and MMAs, frees its TMEM and returns.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <mutex>

namespace cek {
namespace gemm {

constexpr int BM = 128, BK = 128;  // BK in bytes: 128 e4m3 or 64 fp16/bf16 elements

// Operand kinds: e4m3 x e4m3 (tcgen05 kind::f8f6f4), fp16 x fp16 and
// bf16 x bf16 (kind::f16), and fp16 / bf16 activations against FP8 weights
// converted in shared memory (kF16W8 / kBF16W8: kind::f16 MMAs on the
// converted tile).  All K-major, fp32 accumulation.
enum Kind { kE4M3 = 0, kF16 = 1, kBF16 = 2, kF16W8 = 3, kBF16W8 = 4 };
__host__ __device__ constexpr bool is_w8(int k) { return k == kF16W8 || k == kBF16W8; }
// the kind whose MMA runs: W8 kinds multiply the converted 16-bit tile
__host__ __device__ constexpr int mma_kind(int k) { return k == kF16W8 ? kF16 : k == kBF16W8 ? kBF16 : k; }
constexpr int TMEM_COLS = 512;     // two accumulators of up to 256 fp32 columns
constexpr int kSmemBudget = 227 * 1024;

// Tile-N dependent constants.  BN is a multiple of 32 in [128, 256]; the
// stage count fills the shared-memory budget.
template <int BN, int KIND>
struct Tile {
  // W8 kinds add the FP8 staging tile (BN rows x 64 bytes) that the
  // converter warps turn into the 16-bit B tile
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, Q_BYTES = is_w8(KIND) ? BN * 64 : 0;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + Q_BYTES;
  // warps: 0 TMA producer, 1 MMA, 2-5 epilogue, 6-9 converters (W8 kinds)
  static constexpr int THREADS = (is_w8(KIND) ? 10 : 6) * 32;
  // The e4m3 kind stores its output through shared memory with TMA: one
  // 32-row x 16-column staging buffer (1 KB) per epilogue warp, after the ring.
  static constexpr bool TSTORE = KIND == kE4M3;
  static constexpr int EPI_BYTES = TSTORE ? 4 * 1024 : 0;
  static constexpr int STAGES = (kSmemBudget - 2048 - EPI_BYTES) / STAGE_BYTES > 6
                                    ? 6 : (kSmemBudget - 2048 - EPI_BYTES) / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024;  // + alignment slack
  // fp32 accumulate (bit 4), A/B format (bits 7-9 / 10-12: e4m3 = 0 for
  // kind::f8f6f4; f16 = 0, bf16 = 1 for kind::f16), both K-major, N = BN, M = 128
  static constexpr uint32_t FMT = mma_kind(KIND) == kBF16 ? 1u : 0u;
  static constexpr uint32_t IDESC =
      (1u << 4) | (FMT << 7) | (FMT << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
};
constexpr uint32_t kWaitPolls = 1u << 24;

__device__ unsigned long long g_timeouts;

CEK_DEVICE uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CEK_DEVICE bool try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait; false means it gave up.
CEK_DEVICE bool wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *abort_flag) return false;
  }
  *abort_flag = 1;
  atomicAdd(&g_timeouts, 1ull);
  return false;
}
CEK_DEVICE void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
CEK_DEVICE void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
CEK_DEVICE void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
CEK_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}
// TMA tensor store of a staged tile (bulk-group completion), and its waits
CEK_DEVICE void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(map), "r"(x), "r"(y), "r"(src) : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
CEK_DEVICE void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
CEK_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
CEK_DEVICE void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CEK_DEVICE void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand, rows of 128 bytes with
// the 128-byte swizzle, 8-row core groups 1024 bytes apart.
CEK_DEVICE uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);        // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                         // 128-byte swizzle
  return d;
}
template <int KIND>
CEK_DEVICE void mma_issue(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == kE4M3)
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
  else
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
CEK_DEVICE void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

CEK_DEVICE void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct Params {
  const float* a_scale;  // per-row [M], or null (1.0)
  const float* b_scale;  // per-column [N], or a scalar when b_scalar
  void* y;
  int M, N, K;
  int num_m, num_n;
  int kblocks;           // K bytes / BK
  int kblock_elems;      // elements per k-block (TMA x step)
  int b_scalar;
};

template <typename OutT, int BN, int KIND, int WFMT = 0>
__global__ void __launch_bounds__(Tile<BN, KIND>::THREADS, 1)
gemm_fp8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_y, const Params p) {
  using TL = Tile<BN, KIND>;
  constexpr int STAGES = TL::STAGES, STAGE_BYTES = TL::STAGE_BYTES, A_BYTES = TL::A_BYTES, B_BYTES = TL::B_BYTES;
  constexpr bool W8 = is_w8(KIND);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], conv_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.num_m * p.num_n;
  const int kblocks = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(saddr(&full_bar[s]), 1);
      bar_init(saddr(&empty_bar[s]), 1);
      bar_init(saddr(&conv_bar[s]), 4);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(saddr(&acc_full[b]), 1);
      bar_init(saddr(&acc_empty[b]), 4);
    }
    bar_init(saddr(&drain_bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(&tmem_base_sh)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      pdl_wait();
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && !abort_flag; t += gridDim.x) {
        const int mb = t % p.num_m, nb = t / p.num_m;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait(saddr(&empty_bar[s]), ((it / STAGES) & 1) ^ 1, &abort_flag)) break;
          uint8_t* sa = smem + s * STAGE_BYTES;
          const uint32_t fb = saddr(&full_bar[s]);
          if constexpr (W8) {
            // A (16-bit, swizzled) and the FP8 weight tile into the staging area
            bar_expect_tx(fb, A_BYTES + TL::Q_BYTES);
            tma_load_2d(saddr(sa), &map_a, kb * p.kblock_elems, mb * BM, fb);
            tma_load_2d(saddr(sa + A_BYTES + B_BYTES), &map_b, kb * p.kblock_elems, nb * BN, fb);
          } else {
            bar_expect_tx(fb, STAGE_BYTES);
            tma_load_2d(saddr(sa), &map_a, kb * p.kblock_elems, mb * BM, fb);
            tma_load_2d(saddr(sa + A_BYTES), &map_b, kb * p.kblock_elems, nb * BN, fb);
          }
        }
      }
      // Before leaving, make sure no copy of ours is still landing (bounded).
      for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        wait(saddr(&full_bar[j % STAGES]), (j / STAGES) & 1, &abort_flag);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int it = 0, local = 0;
      for (int t = blockIdx.x; t < num_tiles && !abort_flag; t += gridDim.x, ++local) {
        const int b = local & 1;
        if (!wait(saddr(&acc_empty[b]), ((local >> 1) & 1) ^ 1, &abort_flag)) break;
        fence_after();
        const uint32_t d = tmem_base + b * 256;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          // W8: the converters' barrier (they waited for the copies first)
          if (!wait(saddr(W8 ? &conv_bar[s] : &full_bar[s]), (it / STAGES) & 1, &abort_flag)) { ok = false; break; }
          fence_after();
          const uint32_t a0 = saddr(smem + s * STAGE_BYTES), b0 = a0 + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_issue<mma_kind(KIND)>(d, smem_desc(a0 + k * 32), smem_desc(b0 + k * 32), TL::IDESC,
                                      (kb | k) ? 1u : 0u);
          mma_commit(saddr(&empty_bar[s]));
        }
        if (!ok) break;
        mma_commit(saddr(&acc_full[b]));
      }
      // All MMAs of this thread finished before TMEM is released (bounded).
      mma_commit(saddr(&drain_bar));
      wait(saddr(&drain_bar), 0, &abort_flag);
    }
  } else if (W8 && warp >= 6) {
    // ---------------- converters (warps 6..9, W8 kinds) ----------------
    // FP8 staging tile (BN rows x 64 bytes, dense) -> 16-bit B tile in the
    // layout a 128-byte-swizzled TMA copy would leave: row r at 128 r, 16-byte
    // chunk j at chunk position j ^ (r & 7).  Exact conversion.
    const int ct = threadIdx.x - 6 * 32;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles && !abort_flag; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const int s = it % STAGES;
        if (!wait(saddr(&full_bar[s]), (it / STAGES) & 1, &abort_flag)) { ok = false; break; }
        const uint32_t bt = saddr(smem + s * STAGE_BYTES) + A_BYTES, qt = bt + B_BYTES;
        for (int u = ct; u < BN * 2; u += 128) {
          const int r = u >> 1, h = u & 1;
          uint4 q[2];
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(q[0].x), "=r"(q[0].y), "=r"(q[0].z), "=r"(q[0].w)
                       : "r"(qt + r * 64 + h * 32));
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(q[1].x), "=r"(q[1].y), "=r"(q[1].z), "=r"(q[1].w)
                       : "r"(qt + r * 64 + h * 32 + 16));
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t w0 = (c & 1) ? q[c >> 1].z : q[c >> 1].x, w1 = (c & 1) ? q[c >> 1].w : q[c >> 1].y;
            uint32_t o[4];
            if constexpr (mma_kind(KIND) == kF16) {
              o[0] = fp8x2_to_f16x2<WFMT, 0>(w0); o[1] = fp8x2_to_f16x2<WFMT, 1>(w0);
              o[2] = fp8x2_to_f16x2<WFMT, 0>(w1); o[3] = fp8x2_to_f16x2<WFMT, 1>(w1);
            } else {
              o[0] = fp8x2_to_bf16x2<WFMT, 0>(w0); o[1] = fp8x2_to_bf16x2<WFMT, 1>(w0);
              o[2] = fp8x2_to_bf16x2<WFMT, 0>(w1); o[3] = fp8x2_to_bf16x2<WFMT, 1>(w1);
            }
            const int j = 4 * h + c;
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(bt + r * 128 + ((j ^ (r & 7)) << 4)),
                         "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]) : "memory");
          }
        }
        // the tensor cores read shared memory through the async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive(saddr(&conv_bar[s]));
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    OutT* y = static_cast<OutT*>(p.y);
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles && !abort_flag; t += gridDim.x, ++local) {
      const int b = local & 1;
      const int mb = t % p.num_m, nb = t / p.num_m;
      if (!wait(saddr(&acc_full[b]), (local >> 1) & 1, &abort_flag)) break;
      fence_after();
      const int row = mb * BM + quad * 32 + lane;
      const bool rv = row < p.M;
      const float as = rv ? (p.a_scale ? p.a_scale[row] : 1.f) : 0.f;
      OutT* yrow = y + (size_t)(rv ? row : 0) * p.N;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + b * 256;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        const int n0 = nb * BN + c;
        // the chunk's 32 column scales: one load per lane, then shuffles
        // (warp-uniform control: every lane takes part)
        const float bsv = n0 + lane < p.N ? __ldg(p.b_scale + (p.b_scalar ? 0 : n0 + lane)) : 0.f;
        // N % 16 == 0: the chunk holds 16 or 32 valid columns
        const bool hi = n0 + 16 < p.N;
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float bs0 = __shfl_sync(0xffffffffu, bsv, 2 * i), bs1 = __shfl_sync(0xffffffffu, bsv, 2 * i + 1);
          o[i] = pack2<OutT>(__uint_as_float(r[2 * i]) * as * bs0, __uint_as_float(r[2 * i + 1]) * as * bs1);
        }
        if constexpr (TL::TSTORE) {
          // Through shared memory: lane l writes its row's 16 columns (32 B)
          // at l * 32 of the warp's buffer, then one lane stores the 32 x 16
          // box with TMA (rows >= M are clipped by the tensor map; n0 is a
          // multiple of 16 and N % 16 == 0, so a box is all in or all out).
          // A row per lane over 16-byte stores would touch 32 lines a store.
          const uint32_t buf = saddr(smem + STAGES * STAGE_BYTES + quad * 1024);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (lane == 0) bulk_wait_read_all();  // the previous box has left the buffer
            __syncwarp();
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(buf + lane * 32), "r"(o[8 * h]),
                         "r"(o[8 * h + 1]), "r"(o[8 * h + 2]), "r"(o[8 * h + 3]) : "memory");
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(buf + lane * 32 + 16), "r"(o[8 * h + 4]),
                         "r"(o[8 * h + 5]), "r"(o[8 * h + 6]), "r"(o[8 * h + 7]) : "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0 && n0 + 16 * h < p.N) tma_store_2d(&map_y, buf, n0 + 16 * h, mb * BM + quad * 32);
          }
        } else if (rv && n0 < p.N) {
          uint4* dst = reinterpret_cast<uint4*>(yrow + n0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          if (hi) {
            dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
            dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(saddr(&acc_empty[b]));
    }
    // every staged box written out before the CTA (and its shared memory) ends
    if (TL::TSTORE && lane == 0) bulk_wait_all();
  }

  fence_before();
  __syncthreads();
  fence_after();
  __syncwarp();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
}

// ---- host side ---------------------------------------------------------------------

// ---- the same GEMM on CTA pairs (tcgen05 cta_group::2) ----------------------------
//
// A cluster of two CTAs (one per SM) computes a 256 x BN tile: each CTA loads
// its own 128 rows of A and half of the BN rows of B (BN / 2) with plain TMA
// (no multicast), and the pair's leader (rank 0) issues
// tcgen05.mma.cta_group::2 (M = 256), which reads A and B from both CTAs'
// shared memory and accumulates each CTA's 128 rows into that CTA's TMEM.
// Per SM this halves the B traffic from L2 and the B tile in shared memory
// for the same tile width.
//  * full barriers live in the leader: the leader's producer expects both
//    CTAs' bytes; the peer's loads complete their bytes on the leader's
//    barrier (the cta_group::2 form of the TMA load);
//  * the leader's commits arrive on both CTAs' empty and accumulator-full
//    barriers (commit with .multicast::cluster);
//  * both CTAs' epilogue warps arrive on the leader's accumulator-empty
//    barrier (the peer remotely, through mapa);
//  * TMEM is allocated and freed by warp 1 of each CTA (cta_group::2), and a
//    cluster barrier precedes the free, so no MMA is still writing.
namespace pair {

CEK_DEVICE uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
CEK_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
CEK_DEVICE uint32_t map_to(uint32_t saddr_local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr_local), "r"(rank));
  return r;
}
// bounded wait with cluster-scope acquire (the barrier receives arrivals
// from the peer CTA)
CEK_DEVICE bool wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    if (ok) return true;
    if ((i & 1023u) == 1023u && *abort_flag) return false;
  }
  *abort_flag = 1;
  atomicAdd(&g_timeouts, 1ull);
  return false;
}
CEK_DEVICE void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
CEK_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(leader_bar) : "memory");
}
CEK_DEVICE void mma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p; }"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive on the barrier at this address in both CTAs of the pair
CEK_DEVICE void commit_both(uint32_t bar) {
  asm volatile(
      "{ .reg .b16 m; mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m; }"
      ::"r"(bar) : "memory");
}
CEK_DEVICE void commit_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

template <int BN>
struct PairTile {
  static constexpr int A_BYTES = BM * BK, B_BYTES = (BN / 2) * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int THREADS = 6 * 32;
  static constexpr int STAGES = (kSmemBudget - 2048) / STAGE_BYTES > 8 ? 8 : (kSmemBudget - 2048) / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
  // e4m3 x e4m3, fp32 accumulate, K-major, N = BN, M = 256 (the pair)
  static constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(256 >> 4) << 24);
};

template <typename OutT, int BN>
__global__ void __launch_bounds__(PairTile<BN>::THREADS, 1)
gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const Params p) {
  using TL = PairTile<BN>;
  constexpr int STAGES = TL::STAGES, STAGE_BYTES = TL::STAGE_BYTES, A_BYTES = TL::A_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_m2 = (p.M + 2 * BM - 1) / (2 * BM);
  const int num_tiles = num_m2 * p.num_n;
  const int kblocks = p.kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      bar_init(saddr(&full_bar[s]), 1);
      bar_init(saddr(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(saddr(&acc_full[b]), 1);
      bar_init(saddr(&acc_empty[b]), 8);  // both CTAs' four epilogue warps (used in the leader)
    }
    bar_init(saddr(&drain_bar), 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base_sh)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  cluster_sync();
  fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      pdl_wait();
      int it = 0;
      for (int t = cluster; t < num_tiles && !abort_flag; t += nclusters) {
        const int mb = t % num_m2, nb = t / num_m2;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait(saddr(&empty_bar[s]), ((it / STAGES) & 1) ^ 1, &abort_flag)) break;
          uint8_t* sa = smem + s * STAGE_BYTES;
          const uint32_t fb = map_to(saddr(&full_bar[s]), 0);
          if (leader) bar_expect_tx(saddr(&full_bar[s]), 2 * STAGE_BYTES);
          tma_load_2d_pair(saddr(sa), &map_a, kb * p.kblock_elems, mb * 2 * BM + (int)rank * BM, fb);
          tma_load_2d_pair(saddr(sa + A_BYTES), &map_b, kb * p.kblock_elems, nb * BN + (int)rank * (BN / 2), fb);
        }
      }
      // before leaving: our copies have landed once the MMAs that read the
      // last stages committed (their empty barriers; bounded)
      for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        wait(saddr(&empty_bar[j % STAGES]), (j / STAGES) & 1, &abort_flag);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (lane == 0 && leader) {
      int it = 0, local = 0;
      for (int t = cluster; t < num_tiles && !abort_flag; t += nclusters, ++local) {
        const int b = local & 1;
        if (!wait_cluster(saddr(&acc_empty[b]), ((local >> 1) & 1) ^ 1, &abort_flag)) break;
        fence_after();
        const uint32_t d = tmem_base + b * 256;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!wait_cluster(saddr(&full_bar[s]), (it / STAGES) & 1, &abort_flag)) { ok = false; break; }
          fence_after();
          const uint32_t a0 = saddr(smem + s * STAGE_BYTES), b0 = a0 + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_pair(d, smem_desc(a0 + k * 32), smem_desc(b0 + k * 32), TL::IDESC, (kb | k) ? 1u : 0u);
          commit_both(saddr(&empty_bar[s]));
        }
        if (!ok) break;
        commit_both(saddr(&acc_full[b]));
      }
      commit_local(saddr(&drain_bar));
      wait(saddr(&drain_bar), 0, &abort_flag);
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    pdl_wait();
    const int quad = warp & 3;
    OutT* y = static_cast<OutT*>(p.y);
    const uint32_t leader_empty[2] = {map_to(saddr(&acc_empty[0]), 0), map_to(saddr(&acc_empty[1]), 0)};
    int local = 0;
    for (int t = cluster; t < num_tiles && !abort_flag; t += nclusters, ++local) {
      const int b = local & 1;
      const int mb = t % num_m2, nb = t / num_m2;
      if (!wait(saddr(&acc_full[b]), (local >> 1) & 1, &abort_flag)) break;
      fence_after();
      const int row = mb * 2 * BM + (int)rank * BM + quad * 32 + lane;
      const bool rv = row < p.M;
      const float as = rv ? p.a_scale[row] : 0.f;
      OutT* yrow = y + (size_t)(rv ? row : 0) * p.N;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + b * 256;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        const int n0 = nb * BN + c;
        const float bsv = n0 + lane < p.N ? __ldg(p.b_scale + n0 + lane) : 0.f;
        const bool hi = n0 + 16 < p.N;
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float bs0 = __shfl_sync(0xffffffffu, bsv, 2 * i), bs1 = __shfl_sync(0xffffffffu, bsv, 2 * i + 1);
          o[i] = pack2<OutT>(__uint_as_float(r[2 * i]) * as * bs0, __uint_as_float(r[2 * i + 1]) * as * bs1);
        }
        if (rv && n0 < p.N) {
          uint4* dst = reinterpret_cast<uint4*>(yrow + n0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          if (hi) {
            dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
            dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) arrive_remote(leader_empty[b]);
    }
  }

  fence_before();
  __syncwarp();
  cluster_sync();
  fence_after();
  __syncwarp();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
}

}  // namespace pair

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Row-major [rows, cols] matrix of `eb`-byte elements; box = box_bytes of a
// row (one k-block) x box_rows rows (box_rows <= 256, the TMA box limit),
// 128-byte swizzle unless `dense` (the W8 staging tile).
bool encode_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int eb,
                int box_bytes, bool dense) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * eb)};
  cuuint32_t box[2] = {(cuuint32_t)(box_bytes / eb), (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, eb == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base),
             dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             dense ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encoded maps of recent calls, keyed by everything the encoding reads.  A
// layer calls the GEMM with the same weight (and usually the same activation
// buffer) every step, so the host-side encode runs once per buffer instead of
// once per call.  A map holds only the address and the shape; a buffer freed
// and reallocated at the same address with the same shape encodes identically.
struct MapKey {
  const void* base;
  int64_t rows, cols;
  int box_rows, eb, box_bytes;
  bool dense;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && box_rows == o.box_rows && eb == o.eb &&
           box_bytes == o.box_bytes && dense == o.dense;
  }
};
constexpr int kMapCacheSize = 64;
struct MapCache {
  std::mutex mu;
  MapKey key[kMapCacheSize];
  CUtensorMap map[kMapCacheSize];
  int used = 0, next = 0;
};

bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows, int eb = 1,
              int box_bytes = BK, bool dense = false) {
  static MapCache cache;
  const MapKey k{base, rows, cols, box_rows, eb, box_bytes, dense};
  {
    std::lock_guard<std::mutex> g(cache.mu);
    for (int i = 0; i < cache.used; ++i)
      if (cache.key[i] == k) {
        *m = cache.map[i];
        return true;
      }
  }
  if (!encode_map(m, base, rows, cols, box_rows, eb, box_bytes, dense)) return false;
  std::lock_guard<std::mutex> g(cache.mu);
  const int slot = cache.used < kMapCacheSize ? cache.used++ : (cache.next++ % kMapCacheSize);
  cache.key[slot] = k;
  cache.map[slot] = *m;
  return true;
}

template <typename OutT, int BN, int KIND, int WFMT = 0>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& my, const Params& p, cudaStream_t st) {
  auto kern = gemm_fp8_kernel<OutT, BN, KIND, WFMT>;
  constexpr int SMEM_BYTES = Tile<BN, KIND>::SMEM_BYTES;
  static cek_host::DeviceSlots attr_set;
  const int sms = cek_host::sm_count();
  if (!cek_host::ensure_smem_attr(attr_set, kern, SMEM_BYTES)) return CEK_ERR_LAUNCH;
  const int tiles = p.num_m * p.num_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles < sms ? tiles : sms));
  cfg.blockDim = dim3(Tile<BN, KIND>::THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, my, p) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

template <typename OutT, int BN>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t st) {
  auto kern = pair::gemm_fp8_pair_kernel<OutT, BN>;
  constexpr int SMEM_BYTES = pair::PairTile<BN>::SMEM_BYTES;
  static cek_host::DeviceSlots attr_set;
  const int sms = cek_host::sm_count();
  if (!cek_host::ensure_smem_attr(attr_set, kern, SMEM_BYTES)) return CEK_ERR_LAUNCH;
  const int tiles = ((p.M + 2 * BM - 1) / (2 * BM)) * p.num_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sms);
  cfg.blockDim = dim3(pair::PairTile<BN>::THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // as many pairs as can be resident at once (SM pairs within a GPC), once per device
  static cek_host::DeviceSlots max_pairs;
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>* slot = max_pairs.at(dev);
  int mp = slot ? slot->load() : 0;
  if (mp <= 0) {
    cfg.gridDim = dim3((unsigned)sms);
    if (cudaOccupancyMaxActiveClusters(&mp, kern, &cfg) != cudaSuccess || mp <= 0) mp = sms / 2;
    if (slot) slot->store(mp);
  }
  const int pairs = std::min(tiles, std::min(mp, sms / 2));
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, p) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

// CTA-pair path: CEK_GEMM_PAIR=1 turns it on (per-token FP8 GEMM, M > 128).
// Off by default: at N = 14336, K = 4096 it measured 106.9 / 365.0 us at
// M = 2048 / 8192 against 102.4 / 353.3 us for the one-CTA kernel (tensor
// pipe 55.5 % against 59.9 % of elapsed; L2 at 37-42 % of its peak, so the
// halved B traffic buys nothing here).
bool use_pair(int64_t M) {
  static const int mode = [] {
    const char* v = std::getenv("CEK_GEMM_PAIR");
    return v ? std::atoi(v) : 0;
  }();
  return mode == 1 && M > BM;
}

// Tile N for the pair path: as choose_bn over 256-row tiles and SM pairs.
int choose_bn_pair(int64_t M, int64_t N) {
  const int pairs = cek_host::sm_count() / 2;  // (the resident pairs are at most this)
  const int64_t num_m2 = (M + 2 * BM - 1) / (2 * BM);
  const int cands[4] = {256, 224, 192, 160};
  int bn = 256;
  int64_t best = INT64_MAX / 100;
  for (int c : cands) {
    const int64_t tiles = num_m2 * ((N + c - 1) / c);
    const int64_t cost = ((tiles + pairs - 1) / pairs) * c;
    if (cost * 100 < best * 97) { best = cost; bn = c; }
  }
  return bn;
}

int run_pair(const void* a, const void* b, const float* a_scale, const float* b_scale, void* y, int64_t M,
             int64_t N, int64_t K, int y_dtype, cudaStream_t st) {
  const int bn = choose_bn_pair(M, N);
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, M, K, BM) || !make_map(&mb, b, N, K, bn / 2)) return CEK_ERR_LAUNCH;
  Params p;
  p.a_scale = a_scale; p.b_scale = b_scale; p.y = y;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.num_m = (int)((M + BM - 1) / BM);
  p.num_n = (int)((N + bn - 1) / bn);
  p.kblocks = (int)(K / BK);
  p.kblock_elems = BK;
  p.b_scalar = 0;
#define CEK_GEMM_PAIR_BN(B)                                                               \
  if (bn == B) return y_dtype == CEK_F16 ? launch_pair<__half, B>(ma, mb, p, st)         \
                                         : launch_pair<__nv_bfloat16, B>(ma, mb, p, st);
  CEK_GEMM_PAIR_BN(256) CEK_GEMM_PAIR_BN(224) CEK_GEMM_PAIR_BN(192) CEK_GEMM_PAIR_BN(160)
#undef CEK_GEMM_PAIR_BN
  return CEK_ERR_UNSUPPORTED;
}

int choose_bn(int64_t M, int64_t N, bool e4m3) {
  // Tile N for the e4m3 kind: the candidate with the fewest rounds of tiles
  // over the SMs, the widest on a tie.  Its tiles cost about the same whatever
  // their width (per 128-byte k-block ~0.41 us at K = 4096, measured at
  // M = 2048 / 8192: 13-14.4 us a tile for BN = 160-256), so only the rounds
  // count: at M = 2048, N = 14336 BN = 256 (7 rounds, the last nearly empty)
  // 99.3 us, 224 (7 rounds) 100.8, 192 (9) 117.3, 160 (10) 129.5.
  // The 16-bit kinds minimise rounds x BN, a narrower tile having to win by
  // more than 3 %.
  const int sms = cek_host::sm_count();
  const int64_t num_m = (M + BM - 1) / BM;
  const int cands[4] = {256, 224, 192, 160};
  int bn = 256;
  int64_t best = INT64_MAX / 100;
  for (int c : cands) {
    const int64_t tiles = num_m * ((N + c - 1) / c);
    const int64_t rounds = (tiles + sms - 1) / sms;
    if (e4m3) {
      if (rounds < best) { best = rounds; bn = c; }
    } else if (rounds * c * 100 < best * 97) {
      best = rounds * c;
      bn = c;
    }
  }
  static const int bn_env = [] {  // CEK_GEMM_BN forces the tile N (tuning only)
    const char* v = std::getenv("CEK_GEMM_BN");
    return v ? std::atoi(v) : 0;
  }();
  if (bn_env == 256 || bn_env == 224 || bn_env == 192 || bn_env == 160) bn = bn_env;
  return bn;
}

// Builds the maps and launches: a [M, K] and b [N, K], elements of `eb` bytes.
template <int KIND, int WFMT = 0>
int run(const void* a, const void* b, const float* a_scale, const float* b_scale, bool b_scalar, void* y,
        int64_t M, int64_t N, int64_t K, int eb, int y_dtype, cudaStream_t st) {
  const int bn = choose_bn(M, N, KIND == kE4M3);
  CUtensorMap ma, mb;
  // W8 kinds: b is the FP8 weight, copied as dense 64-byte x bn boxes (one
  // k-block of 64 elements) into the staging tile
  const bool bmap = is_w8(KIND) ? make_map(&mb, b, N, K, bn, 1, 64, true) : make_map(&mb, b, N, K, bn, eb);
  if (!make_map(&ma, a, M, K, BM, eb) || !bmap) return CEK_ERR_LAUNCH;
  // the output's map (e4m3 kind): 16-bit elements, 16 x 32 boxes, no swizzle
  CUtensorMap my = ma;
  if (Tile<256, KIND>::TSTORE && !make_map(&my, y, M, N, 32, 2, 32, true)) return CEK_ERR_LAUNCH;
  Params p;
  p.a_scale = a_scale; p.b_scale = b_scale; p.y = y;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.num_m = (int)((M + BM - 1) / BM);
  p.num_n = (int)((N + bn - 1) / bn);
  p.kblocks = (int)(K * eb / BK);
  p.kblock_elems = BK / eb;
  p.b_scalar = b_scalar ? 1 : 0;
#define CEK_GEMM_BN(B)                                                                        \
  if (bn == B) return y_dtype == CEK_F16 ? launch<__half, B, KIND, WFMT>(ma, mb, my, p, st)      \
                                         : launch<__nv_bfloat16, B, KIND, WFMT>(ma, mb, my, p, st);
  CEK_GEMM_BN(256) CEK_GEMM_BN(224) CEK_GEMM_BN(192) CEK_GEMM_BN(160)
#undef CEK_GEMM_BN
  return CEK_ERR_UNSUPPORTED;
}

// Exact FP8 -> 16-bit dequantisation of a weight matrix (8 codes per thread).
template <typename T, int FMT>
__global__ void __launch_bounds__(256) dequant_fp8_kernel(const uint8_t* __restrict__ w, T* __restrict__ out,
                                                          int64_t n8) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint2 v = reinterpret_cast<const uint2*>(w)[i];
  uint32_t o[4];
  const uint32_t words[2] = {v.x, v.y};
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if constexpr (std::is_same<T, __half>::value) {
      o[2 * q] = fp8x2_to_f16x2<FMT>(words[q] & 0xFFFFu);
      o[2 * q + 1] = fp8x2_to_f16x2<FMT>(words[q] >> 16);
    } else {
      o[2 * q] = fp8x2_to_bf16x2<FMT>(words[q] & 0xFFFFu);
      o[2 * q + 1] = fp8x2_to_bf16x2<FMT>(words[q] >> 16);
    }
  }
  reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace gemm
}  // namespace cek

extern "C" int cek_gemm_fp8_scaled(const void* aq, const void* bq, const float* a_scale,
                                   const float* b_scale, void* y, int64_t M, int64_t N, int64_t K,
                                   int y_dtype, void* stream) {
  using namespace cek::gemm;
  if (M < 0 || N < 0 || K < 0) return CEK_ERR_INVALID_ARG;
  if (y_dtype != CEK_F16 && y_dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CEK_OK;
  if (K == 0 || K % BK != 0 || N % 16 != 0) return CEK_ERR_INVALID_ARG;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return CEK_ERR_INVALID_ARG;
  if (!aq || !bq || !a_scale || !b_scale || !y) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(aq) || !cek_host::aligned16(bq) || !cek_host::aligned16(y))
    return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cek::gemm::use_pair(M)) return cek::gemm::run_pair(aq, bq, a_scale, b_scale, y, M, N, K, y_dtype, st);
  return cek::gemm::run<cek::gemm::kE4M3>(aq, bq, a_scale, b_scale, false, y, M, N, K, 1, y_dtype, st);
}

extern "C" int64_t cek_gemm_fp8w_workspace_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return ((N * K * 2 + 255) / 256) * 256;
}

// Up to this many tokens the weight tile is converted inside the GEMM (each
// tile once per 128-row block: cheap while there are few); above it the
// weight is dequantised once into the workspace and the plain 16-bit GEMM
// runs.  Measured at N = 14336, K = 4096: in-kernel 34.9 / 46.6 / 86.0 us at
// M = 128 / 256 / 512 against 61.9 / 64.7 / 87.2 us dequantise-first, and
// 283 against 206 us at M = 2048.
constexpr int64_t kGemmW8MaxRows = CEK_GEMM_FP8W_INKERNEL_MAX_ROWS;

// GEMV family or this GEMM for 17..256 tokens, by estimated time (B200, CUDA
// graph of calls over cold weights, per-tensor scale):
//  * GEMV family: ~1.55e-8 us per weight byte per token + 8 us (14336 x 4096:
//    M = 32 / 64 / 128 took 35.3 / 62.5 / 118.5 us; 6144 x 4096: 21.4 / 36.8
//    / 67.0 us);
//  * this GEMM: rounds of its 128 x 256 tiles over the SMs x 7.8 us per 1024
//    of K (14336 x 4096: 32 us at any M in 17..128; 6144 x 4096: 31 us;
//    4096 x 14336, 16 tiles on 16 SMs: 95 us at any M).
// So 14336 x 4096 moves to the GEMM from M = 26, 6144 x 4096 from M = 60 and
// 4096 x 14336 from M = 112 (28672 x 4096 from M = 17).
extern "C" int cek_gemm_fp8w_preferred(int64_t M, int64_t N, int64_t K) {
  if (M <= 16 || N <= 0 || K <= 0 || K % 64 != 0 || N % 16 != 0) return 0;
  if (M > kGemmW8MaxRows) return 1;
  const int64_t sms = cek_host::sm_count();
  const int64_t tiles = ((M + 127) / 128) * ((N + 255) / 256);
  const double gemm_us = (double)((tiles + sms - 1) / sms) * 7.8 * (double)K / 1024.0;
  const double gemv_us = 1.55e-8 * (double)N * (double)K * (double)M + 8.0;
  return gemm_us < gemv_us ? 1 : 0;
}

extern "C" int cek_gemm_fp8w(const void* x, const void* w, const void* scale, void* y, void* workspace,
                             int64_t workspace_bytes, int64_t M, int64_t N, int64_t K, int dtype, int w_fmt,
                             int scale_kind, void* stream) {
  using namespace cek::gemm;
  if (M < 0 || N < 0 || K < 0 || workspace_bytes < 0) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind != CEK_SCALE_PERN_F32 && scale_kind != CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return CEK_OK;
  if (K == 0 || K % 64 != 0 || N % 16 != 0) return CEK_ERR_INVALID_ARG;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return CEK_ERR_INVALID_ARG;
  // the workspace is used (and required) only above kGemmW8MaxRows tokens
  const bool need_ws = M > kGemmW8MaxRows;
  if (!x || !w || !scale || !y || (need_ws && !workspace)) return CEK_ERR_INVALID_ARG;
  if (need_ws && workspace_bytes < cek_gemm_fp8w_workspace_bytes(N, K)) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(x) || !cek_host::aligned16(w) || !cek_host::aligned16(y) ||
      (need_ws && !cek_host::aligned16(workspace)))
    return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float* sc = static_cast<const float*>(scale);
  const bool scalar = scale_kind == CEK_SCALE_PERT_F32;
  if (M <= kGemmW8MaxRows) {
    if (dtype == CEK_F16)
      return w_fmt == CEK_E4M3 ? run<kF16W8, CEK_E4M3>(x, w, nullptr, sc, scalar, y, M, N, K, 2, dtype, st)
                               : run<kF16W8, CEK_E5M2>(x, w, nullptr, sc, scalar, y, M, N, K, 2, dtype, st);
    return w_fmt == CEK_E4M3 ? run<kBF16W8, CEK_E4M3>(x, w, nullptr, sc, scalar, y, M, N, K, 2, dtype, st)
                             : run<kBF16W8, CEK_E5M2>(x, w, nullptr, sc, scalar, y, M, N, K, 2, dtype, st);
  }
  const int64_t n8 = N * K / 8;
  const unsigned blocks = (unsigned)((n8 + 255) / 256);
  const uint8_t* wq = static_cast<const uint8_t*>(w);
#define CEK_DQ(T, F) cek::gemm::dequant_fp8_kernel<T, F><<<blocks, 256, 0, st>>>(wq, static_cast<T*>(workspace), n8)
  if (dtype == CEK_F16) {
    if (w_fmt == CEK_E4M3) CEK_DQ(__half, CEK_E4M3); else CEK_DQ(__half, CEK_E5M2);
  } else {
    if (w_fmt == CEK_E4M3) CEK_DQ(__nv_bfloat16, CEK_E4M3); else CEK_DQ(__nv_bfloat16, CEK_E5M2);
  }
#undef CEK_DQ
  if (cudaGetLastError() != cudaSuccess) return CEK_ERR_LAUNCH;
  return dtype == CEK_F16
             ? run<kF16>(x, workspace, nullptr, sc, scalar, y, M, N, K, 2, dtype, st)
             : run<kBF16>(x, workspace, nullptr, sc, scalar, y, M, N, K, 2, dtype, st);
}

extern "C" int cek_gemm_fp8_timeouts(uint64_t* count) {
  if (!count) return CEK_ERR_INVALID_ARG;
  unsigned long long v = 0;
  if (cudaMemcpyFromSymbol(&v, cek::gemm::g_timeouts, sizeof(v)) != cudaSuccess) return CEK_ERR_LAUNCH;
  *count = v;
  return CEK_OK;
}
