// tp_allreduce.cu — the row-parallel FP8 GEMV fused with its all-reduce over
// NVLink peer memory, for the tensor-parallel decode step.
//
//   out[m, n] = sum over ranks r of GEMV_r(x_r, w_r)[m, n]
//
// Two launches per call:
//  1. The split-K GEMV of gemv_fp8.cu in push mode: every CTA stores its
//     finished output tile straight into slot `rank` of every rank's receive
//     buffer (plain stores through CUDA IPC mappings over NVLink), so the
//     transfer overlaps the remaining tiles' math.  The GEMV itself neither
//     fences nor signals (a per-CTA system fence and arrival counter cost
//     ~15 us: every CTA held its slot until its remote stores were acked).
//  2. tp_reduce_kernel (programmatic launch; griddepcontrol.wait returns
//     once the GEMV has completed, i.e. all its pushes are performed): one
//     thread fences at system scope and raises this rank's ready flag,
//     stamped with the call's epoch, on every rank (st.release.sys); all CTAs
//     wait (bounded) until every rank's flag shows this epoch, add the
//     receive slots in rank order (fp32, one rounding: every rank computes the
//     same bits) and write `out`; the last CTA advances the epoch.
// Receive slots come in two sets, chosen by epoch parity.  A rank passes the
// ready wait of call e only after every rank has started call e's reduce,
// i.e. finished reading call e-1's set, so call e+1's pushes (into that
// set) never overwrite data still being read: no second barrier is needed.
// The epoch lives in device memory, so a CUDA graph replaying the pair stays
// correct.  No TMA, no multicast: peers are reached with ordinary loads and
// stores.  A wait that runs out sets bit 0 of the sync block's error word
// (cek_comm_errors) and the kernel carries on.
#include "gemv.cuh"

#include <algorithm>
#include <cstring>

namespace cek {
namespace tp {

constexpr long long kWaitPolls = 1ll << 24;

CEK_DEVICE bool wait_at_least(const unsigned* flag, unsigned e, unsigned* errors) {
  for (long long i = 0; i < kWaitPolls; ++i) {
    if ((int)(ld_acquire_sys(flag) - e) >= 0) return true;
    __nanosleep(64);
  }
  atomicOr(errors, 1u);
  return false;
}

template <typename T>
__global__ void __launch_bounds__(256)
tp_reduce_kernel(const unsigned long long* peers, unsigned* sync, T* out, int mn, int rank, int world) {
  // the next kernel may launch now (it waits for this one before reading out)
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&sync[kEpoch]) + 1;
  if (blockIdx.x == 0 && threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned*>(peers[threadIdx.x]) + kReady + rank, e);
  }
  if (threadIdx.x < world) wait_at_least(&sync[kReady + threadIdx.x], e, &sync[kErrors]);
  __syncthreads();
  const T* recv = reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(sync) + kSyncBytes) +
                 (size_t)(e & 1u) * world * mn;
  const int stride = gridDim.x * blockDim.x;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += stride) {
    float v = 0.f;
    for (int r = 0; r < world; ++r) {
      const unsigned short bits = __ldcg(reinterpret_cast<const unsigned short*>(recv) + (size_t)r * mn + i);
      T t;
      *reinterpret_cast<unsigned short*>(&t) = bits;
      v += to_f32<T>(t);
    }
    out[i] = from_f32<T>(v);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&sync[kReduceCount], 1u);
    if (prev == gridDim.x - 1) {
      sync[kReduceCount] = 0;
      *reinterpret_cast<volatile unsigned*>(&sync[kEpoch]) = e;
    }
  }
}

// Barrier over the ranks' comm regions: once every earlier kernel on this
// stream has completed (griddepcontrol.wait), one fence at system scope, this
// rank's ready flag raised on every rank with the call's epoch, a bounded
// wait for every rank's flag, the epoch advanced.  After it, every push made
// by any rank before its own barrier is visible here.
__global__ void __launch_bounds__(32) tp_barrier_kernel(const unsigned long long* peers, unsigned* sync, int rank,
                                                       int world) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&sync[kEpoch]) + 1;
  for (int r = threadIdx.x; r < world; r += 32) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<unsigned*>(peers[r]) + kReady + rank, e);
  }
  for (int r = threadIdx.x; r < world; r += 32) wait_at_least(&sync[kReady + r], e, &sync[kErrors]);
  __syncwarp();
  if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(&sync[kEpoch]) = e;
}

}  // namespace tp
}  // namespace cek

extern "C" int64_t cek_tp_comm_bytes(int64_t slot_elems, int world) {
  if (slot_elems <= 0 || world <= 0 || world > cek::tp::kMaxRanks) return 0;
  return cek::tp::kSyncBytes + 2 * (int64_t)world * slot_elems * 2;  // two slot sets
}

extern "C" int cek_comm_alloc(int64_t bytes, void** ptr) {
  if (bytes <= 0 || !ptr) return CEK_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return CEK_ERR_LAUNCH;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) {
    cudaFree(p);
    return CEK_ERR_LAUNCH;
  }
  *ptr = p;
  return CEK_OK;
}

extern "C" int cek_comm_free(void* ptr) {
  return cudaFree(ptr) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

extern "C" int cek_ipc_get_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return CEK_ERR_INVALID_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == CEK_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return CEK_ERR_LAUNCH;
  memcpy(handle, &h, sizeof(h));
  return CEK_OK;
}

extern "C" int cek_ipc_open_handle(const void* handle, void** ptr) {
  if (!ptr || !handle) return CEK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? CEK_OK
                                                                                       : CEK_ERR_LAUNCH;
}

extern "C" int cek_ipc_close_handle(void* ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

extern "C" int cek_comm_errors(void* my_comm, uint32_t* out) {
  if (!my_comm || !out) return CEK_ERR_INVALID_ARG;
  unsigned v = 0;
  if (cudaMemcpy(&v, static_cast<unsigned*>(my_comm) + cek::tp::kErrors, 4, cudaMemcpyDeviceToHost) !=
      cudaSuccess)
    return CEK_ERR_LAUNCH;
  *out = v;
  return CEK_OK;
}

// Zeroes the whole region (epoch, ready flags, reduce counter, error word,
// slots) and waits for it: the recovery step after a reported timeout, run on
// every rank with no call in flight on any rank.
extern "C" int cek_comm_reset(void* my_comm, int64_t bytes) {
  if (!my_comm || bytes < (int64_t)cek::tp::kSyncBytes) return CEK_ERR_INVALID_ARG;
  if (cudaMemset(my_comm, 0, (size_t)bytes) != cudaSuccess) return CEK_ERR_LAUNCH;
  return cudaDeviceSynchronize() == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}

extern "C" int cek_gemv_fp8_allreduce(const void* x, const void* w, const void* scale, void* out, int64_t M,
                                      int64_t N, int64_t K, int dtype, int w_fmt, int scale_kind,
                                      const uint64_t* peer_comm, void* my_comm, int64_t slot_elems, int rank,
                                      int world, unsigned flags, void* stream) {
  using namespace cek_host;
  if (M <= 0 || N <= 0 || K <= 0 || K % 16 != 0) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (flags & ~(unsigned)CEK_GEMV_EARLY_WEIGHTS) return CEK_ERR_INVALID_ARG;
  if (world < 1 || world > cek::tp::kMaxRanks || rank < 0 || rank >= world) return CEK_ERR_INVALID_ARG;
  if (M * N > slot_elems || M * N > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if (!x || !w || !scale || !out || !peer_comm || !my_comm) return CEK_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(my_comm)) return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cek::GemvParams p = {};
  p.x = x; p.w = static_cast<const uint8_t*>(w); p.scale = scale; p.y = nullptr;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.early_weights = (flags & CEK_GEMV_EARLY_WEIGHTS) ? 1 : 0;
  p.ar_peers = reinterpret_cast<const unsigned long long*>(peer_comm);
  p.ar_sync = static_cast<unsigned*>(my_comm);
  p.ar_rank = rank;
  p.ar_world = world;
  int s = cek::gemv_launch(p, dtype, dtype, w_fmt, scale_kind, false, st);
  if (s != CEK_OK) return s;
  const int mn = (int)(M * N);
  const unsigned blocks = (unsigned)std::min(148, (mn + 255) / 256);
  unsigned* sync = static_cast<unsigned*>(my_comm);
  const unsigned long long* peers = reinterpret_cast<const unsigned long long*>(peer_comm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == CEK_F16)
    e = cudaLaunchKernelEx(&cfg, cek::tp::tp_reduce_kernel<__half>, peers, sync, static_cast<__half*>(out), mn,
                           rank, world);
  else
    e = cudaLaunchKernelEx(&cfg, cek::tp::tp_reduce_kernel<__nv_bfloat16>, peers, sync,
                           static_cast<__nv_bfloat16*>(out), mn, rank, world);
  if (e != cudaSuccess) return CEK_ERR_LAUNCH;
  return launch_status();
}

extern "C" int cek_comm_barrier(const uint64_t* peer_comm, void* my_comm, int rank, int world, void* stream) {
  if (!peer_comm || !my_comm || world < 1 || world > cek::tp::kMaxRanks || rank < 0 || rank >= world)
    return CEK_ERR_INVALID_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, cek::tp::tp_barrier_kernel, reinterpret_cast<const unsigned long long*>(peer_comm),
                         static_cast<unsigned*>(my_comm), rank, world) != cudaSuccess)
    return CEK_ERR_LAUNCH;
  return cek_host::launch_status();
}

extern "C" int cek_gemv_fp8_allgather(const void* x, const void* w, const void* scale, int64_t M, int64_t N,
                                      int64_t K, int64_t row0, int64_t n_full, int64_t y_off, int dtype, int w_fmt,
                                      int scale_kind, const uint64_t* peer_comm, void* my_comm, int64_t comm_bytes,
                                      int rank, int world, unsigned flags, void* stream) {
  using namespace cek_host;
  if (M <= 0 || N <= 0 || K <= 0 || K % 16 != 0 || row0 < 0 || row0 + N > n_full) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (flags & ~(unsigned)CEK_GEMV_EARLY_WEIGHTS) return CEK_ERR_INVALID_ARG;
  if (world < 1 || world > cek::tp::kMaxRanks || rank < 0 || rank >= world) return CEK_ERR_INVALID_ARG;
  if (y_off < 0 || y_off % 2 != 0 || n_full > INT32_MAX || M * n_full > INT32_MAX) return CEK_ERR_INVALID_ARG;
  if ((int64_t)cek::tp::kSyncBytes + y_off + M * n_full * 2 > comm_bytes) return CEK_ERR_INVALID_ARG;
  if (!x || !w || !scale || !peer_comm || !my_comm) return CEK_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w) || !aligned16(my_comm)) return CEK_ERR_ALIGNMENT;
  cek::GemvParams p = {};
  p.x = x; p.w = static_cast<const uint8_t*>(w); p.scale = scale; p.y = nullptr;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.early_weights = (flags & CEK_GEMV_EARLY_WEIGHTS) ? 1 : 0;
  p.ar_peers = reinterpret_cast<const unsigned long long*>(peer_comm);
  p.ar_sync = static_cast<unsigned*>(my_comm);
  p.ar_rank = rank;
  p.ar_world = world;
  p.ag_off = y_off;
  p.ag_n = (int)n_full;
  p.ag_row0 = (int)row0;
  return cek::gemv_launch(p, dtype, dtype, w_fmt, scale_kind, false, static_cast<cudaStream_t>(stream));
}
