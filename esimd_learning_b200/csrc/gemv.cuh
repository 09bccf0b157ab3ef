// gemv.cuh — launch parameters shared by the FP8 GEMV and its fused
// add+RMSNorm prologue variant.
#pragma once
#include "common.cuh"
#include <type_traits>

namespace cek {

constexpr int kMaxMats = 4;  // matrices per multi-GEMV launch

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
  // 1: weights may be streamed before griddepcontrol.wait (the caller
  // guarantees the preceding kernel on the stream does not write them);
  // 0: every global read waits for the preceding kernel.
  int early_weights;
  // 1: gated GeLU output.  w holds 2N rows, gate rows [0, N) then up rows
  // [N, 2N) (scale likewise); y [M, N] = io(gelu_tanh(io(gate)) * io(up))
  // (bulk kernel only)
  int y_gelu;
  // tensor-parallel all-reduce epilogue (ar_world > 0, tp_allreduce.cu):
  // y is pushed into slot ar_rank of every rank's receive buffer instead of
  // being stored to p.y.
  const unsigned long long* ar_peers;  // device array [ar_world] of comm base addresses
  unsigned* ar_sync;                   // this rank's sync block
  int ar_rank, ar_world;
  // several weight matrices sharing x in one launch (nmat > 0): matrix m
  // owns CTAs [mcta_off[m], mcta_off[m+1]) and writes ys[m] [M, ns[m]]
  int nmat;
  const uint8_t* mws[kMaxMats];
  const void* mscales[kMaxMats];
  void* mys[kMaxMats];
  int mns[kMaxMats];
  int mcta_off[kMaxMats + 1];
  // column-parallel all-gather epilogue (ag_n > 0, with ar_world ranks):
  // this call computes rows [ag_row0, ag_row0 + N) of y [M, ag_n] and stores
  // them at byte offset ag_off of the data area of every rank's comm region.
  long long ag_off;
  int ag_n, ag_row0;
  // 1: residual add + RMSNorm prologue inside the bulk GEMV.  x is the
  // hidden state, residual the OLD residual (only read here), gamma the
  // pre-shifted norm weight; every CTA forms io(f32(io(h + r)) * inv_rms *
  // gamma) on chip (shared or tensor memory), inv_rms from the unrounded
  // h + r.  The CTAs trigger their dependents only after their last read of
  // the residual, so a kernel launched behind them may update it in place.
  int norm;
  float eps;
};

// Layout of a rank's tensor-parallel comm region: a 4 KiB sync block
// (32-bit words) followed by two sets of ar_world receive slots of M*N
// elements (set = epoch parity).
namespace tp {
constexpr int kSyncBytes = 4096;
constexpr int kMaxRanks = 64;
constexpr int kReady = 0;        // [kMaxRanks] epoch at which peer r pushed its slot
constexpr int kEpoch = 128;      // last completed epoch of this rank
constexpr int kReduceCount = 130;  // CTAs of the reduce kernel that finished
constexpr int kErrors = 131;     // bit 0: a bounded wait gave up
}  // namespace tp

CEK_DEVICE void st_release_sys(unsigned* addr, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
CEK_DEVICE unsigned ld_acquire_sys(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// ---- device helpers shared by both GEMV kernels ----------------------------------

// Output element (token tok, row n of this call) in one of three modes: a
// local store, the all-reduce push (slot ar_rank of every rank's receive
// buffer, slot set by the call's epoch parity), or the all-gather push (row
// ag_row0 + n of every rank's full output).
// The two push modes, kept out of line and given the fields by value: the
// kernels' common path is the local store, and inlining the pushes (or
// letting the parameter block's address escape) slowed the split-K kernel.
template <typename OutT>
__device__ __noinline__ void store_out_push(const unsigned long long* peers, const unsigned* sync, int rank, int world,
                                            long long ag_off, int ag_n, int ag_row0, int M, int N, int tok, int n,
                                            OutT v) {
  if (ag_n > 0) {
    const size_t off = (size_t)tok * ag_n + ag_row0 + n;
    for (int r = 0; r < world; ++r) reinterpret_cast<OutT*>(peers[r] + tp::kSyncBytes + ag_off)[off] = v;
  } else {
    const unsigned set = (*reinterpret_cast<const volatile unsigned*>(&sync[tp::kEpoch]) + 1) & 1u;
    const size_t off = (((size_t)set * world + rank) * M + tok) * N + n;
    for (int r = 0; r < world; ++r) reinterpret_cast<OutT*>(peers[r] + tp::kSyncBytes)[off] = v;
  }
}
template <typename OutT>
CEK_DEVICE void store_out(const GemvParams& p, OutT* y, int ldy, int tok, int n, OutT v) {
  if (p.ar_world == 0) {
    y[(size_t)tok * ldy + n] = v;
  } else if (p.ag_n > 0) {
    const size_t off = (size_t)tok * p.ag_n + p.ag_row0 + n;
    for (int r = 0; r < p.ar_world; ++r)
      reinterpret_cast<OutT*>(p.ar_peers[r] + tp::kSyncBytes + p.ag_off)[off] = v;
  } else {
    const unsigned set = (*reinterpret_cast<volatile unsigned*>(&p.ar_sync[tp::kEpoch]) + 1) & 1u;
    const size_t off = (((size_t)set * p.ar_world + p.ar_rank) * p.M + tok) * p.N + n;
    for (int r = 0; r < p.ar_world; ++r)
      reinterpret_cast<OutT*>(p.ar_peers[r] + tp::kSyncBytes)[off] = v;
  }
}

template <typename InT>
CEK_DEVICE void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);

template <>
CEK_DEVICE void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
CEK_DEVICE void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename InT, int FMT, int HI = 0>
CEK_DEVICE uint32_t cvt_pair(uint32_t pair) {
  if constexpr (std::is_same<InT, __half>::value) return fp8x2_to_f16x2<FMT, HI>(pair);
  else return fp8x2_to_bf16x2<FMT, HI>(pair);
}

template <int SCALE>
CEK_DEVICE float load_scale(const void* s, int n) {
  if constexpr (SCALE == CEK_SCALE_PERN_F16) return __half2float(reinterpret_cast<const __half*>(s)[n]);
  else if constexpr (SCALE == CEK_SCALE_PERN_F32) return reinterpret_cast<const float*>(s)[n];
  else return reinterpret_cast<const float*>(s)[0];
}

// 16 activations of one token at k .. k+15 as 8 packed pairs.
template <typename InT, bool FUSED>
CEK_DEVICE void load_x16(const GemvParams& p, int tok, int k, uint32_t (&xw)[8]) {
  if constexpr (!FUSED) {
    const InT* xp = reinterpret_cast<const InT*>(p.x) + (size_t)tok * p.K + k;
    uint4 a = ldg_nc(xp), b = ldg_nc(xp + 8);
    xw[0] = a.x; xw[1] = a.y; xw[2] = a.z; xw[3] = a.w;
    xw[4] = b.x; xw[5] = b.y; xw[6] = b.z; xw[7] = b.w;
  } else {
    // Residual was written by the preceding stats kernel: plain (coherent) loads.
    const InT* rp = reinterpret_cast<const InT*>(p.residual) + (size_t)tok * p.K + k;
    const InT* gp = reinterpret_cast<const InT*>(p.gamma) + k;
    const uint4* rv = reinterpret_cast<const uint4*>(rp);
    uint4 r0 = rv[0], r1 = rv[1];
    uint4 g0 = ldg_nc(gp), g1 = ldg_nc(gp + 8);
    const float s = p.inv_rms[tok];
    uint32_t rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    uint32_t gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 rf = unpack2<InT>(rr[i]);
      float2 gf = unpack2<InT>(gg[i]);
      xw[i] = pack2<InT>(rf.x * s * gf.x, rf.y * s * gf.y);
    }
  }
}

// Bulk-copy GEMV for up to 16 tokens (gemv_fp8_bulk.cu); CEK_ERR_UNSUPPORTED
// when the call does not fit it.
int gemv_bulk_launch(const GemvParams& p, int x_dtype, int y_dtype, int w_fmt, int scale_kind, cudaStream_t st);

// Plain calls go to gemv_bulk_launch when it accepts them; otherwise (and
// for the fused, multi-matrix and all-reduce variants) the in-CTA split-K
// GEMV (any M, no scratch), launched with PDL on `st`.
int gemv_launch(const GemvParams& base, int x_dtype, int y_dtype, int w_fmt, int scale_kind,
                bool fused, cudaStream_t st);

}  // namespace cek
