// rmsnorm.cu — residual add + RMSNorm, standalone and as the prologue of the
// FP8 GEMV.
//
// Semantics follow FusedAddRmsNorm_batched_kernel
// (csrc/xpu/esimd_kernels/fused_add_rms_norm_batched.h:22-63):
//   pass 1  residual = fp16(hidden + residual), sum of squares over the
//           UNROUNDED fp32 sum                                  (:32-50)
//   pass 2  hidden = fp16(f32(residual_fp16) * inv_rms * w)      (:56-62)
// with inv_rms = rsqrt(sum / K + eps) and w the pre-shifted (w + 1) weight.
//
// B200 layout: one CTA per row, up to 1024 threads, each thread keeps its
// 8..64 elements of the row in registers between the two passes, so the row is read
// once from HBM and written once (the reference re-reads the residual in
// pass 2).  16-byte vector loads/stores; warp-shuffle + shared-memory
// reduction.  Requires K % 8 == 0 and K <= 16384 (the reference requires
// K % 512 == 0).
#include "gemv.cuh"

#include <mutex>
#include <utility>

namespace cek {

constexpr int kNormMaxThreads = 1024;

template <typename T>
CEK_DEVICE float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0.f;
    s = warp_sum(s);
    if (lane == 0) sh[0] = s;
  }
  __syncthreads();
  return sh[0];
}

// What the kernel writes besides the updated residual.
enum NormMode {
  kNormedInPlace = 0,  // standalone op: the normalised row into hidden
  kInvRmsOnly = 1,     // GEMV prologue: the per-row inverse RMS only
  kNormedOut = 2,      // GEMV prologue: the normalised row into a scratch row
};

// VPT = 16-byte vectors per thread.
template <typename T, int VPT, int MODE>
__global__ void __launch_bounds__(kNormMaxThreads)
add_rmsnorm_kernel(T* hidden, T* residual, const T* __restrict__ weight, float* inv_rms_out,
                   T* normed_out, int K, float eps) {
  __shared__ float sh[32];
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  const int nvec = K >> 3;
  uint4* hrow = reinterpret_cast<uint4*>(hidden + (size_t)row * K);
  uint4* rrow = reinterpret_cast<uint4*>(residual + (size_t)row * K);
  uint4 rv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 h = hrow[v], r = rrow[v];
      uint32_t hw[4] = {h.x, h.y, h.z, h.w}, rw[4] = {r.x, r.y, r.z, r.w}, ow[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 hf = unpack2<T>(hw[q]), rf = unpack2<T>(rw[q]);
        const float a = hf.x + rf.x, b = hf.y + rf.y;
        ss += a * a + b * b;
        ow[q] = pack2<T>(a, b);
      }
      rv[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      rrow[v] = rv[i];
    }
  }
  const float total = block_sum<T>(ss, sh);
  const float inv = rsqrtf(total / (float)K + eps);
  if constexpr (MODE == kInvRmsOnly) {
    if (threadIdx.x == 0) inv_rms_out[row] = inv;
  } else {
    uint4* orow = reinterpret_cast<uint4*>((MODE == kNormedInPlace ? hidden : normed_out) + (size_t)row * K);
    const uint4* wv = reinterpret_cast<const uint4*>(weight);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * blockDim.x;
      if (v < nvec) {
        uint4 w4 = wv[v];
        uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
        uint32_t rw[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w}, ow[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 rf = unpack2<T>(rw[q]), wf = unpack2<T>(ww[q]);
          ow[q] = pack2<T>(rf.x * inv * wf.x, rf.y * inv * wf.y);
        }
        orow[v] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
  }
}

template <typename T, int MODE>
static int launch_norm(void* hidden, void* residual, const void* weight, float* inv_rms, void* normed,
                       int64_t rows, int64_t K, float eps, cudaStream_t st) {
  // one 16-byte vector per thread up to 1024 threads, then 2, 4, 8 per thread
  const int nvec = (int)(K / 8);
  const int threads = nvec >= kNormMaxThreads ? kNormMaxThreads : ((nvec + 31) / 32) * 32;
  const int vpt = (nvec + threads - 1) / threads;
  dim3 grid((unsigned)rows), block(threads);
  T* h = static_cast<T*>(hidden);
  T* r = static_cast<T*>(residual);
  const T* w = static_cast<const T*>(weight);
#define CEK_NORM(V)                                                                              \
  if (vpt <= V) {                                                                                \
    return cek_host::launch_pdl(add_rmsnorm_kernel<T, V, MODE>, grid, block, 0, st, h, r, w, inv_rms,   \
                                static_cast<T*>(normed), (int)K, eps);                             \
  }
  CEK_NORM(1) CEK_NORM(2) CEK_NORM(4) CEK_NORM(8)
#undef CEK_NORM
  return CEK_ERR_INVALID_ARG;
}

// residual = io(hidden + residual), launched behind the bulk GEMV with the
// norm prologue.  It may start once every GEMV CTA has read the residual for
// the last time (their programmatic-launch trigger); it triggers its own
// dependents at once and waits for the GEMV's completion before it exits, so
// the next kernel's griddepcontrol.wait covers both.
template <typename T>
__global__ void __launch_bounds__(256) residual_update_kernel(const T* __restrict__ hidden, T* residual, int nvec) {
  pdl_launch_dependents();
  const uint4* hv = reinterpret_cast<const uint4*>(hidden);
  uint4* rv = reinterpret_cast<uint4*>(residual);
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x) {
    const uint4 h = hv[v], r = rv[v];
    const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, rw[4] = {r.x, r.y, r.z, r.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 hf = unpack2<T>(hw[q]), rf = unpack2<T>(rw[q]);
      o[q] = pack2<T>(hf.x + rf.x, hf.y + rf.y);
    }
    rv[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  pdl_wait();
}

// The one-pass fused op: the bulk GEMV forms the normalised rows on chip
// (GemvParams::norm), then residual_update_kernel writes the residual.  No
// scratch memory.  CEK_ERR_UNSUPPORTED when the bulk GEMV cannot hold x on
// chip for this shape (the caller then takes the two-kernel path).
template <typename T>
int fused_norm_gemv_onchip(const void* hidden, void* residual, const void* gamma, float eps, GemvParams p,
                           int dtype, int w_fmt, int scale_kind, cudaStream_t st) {
  static const bool off = [] {
    const char* v = std::getenv("CEK_FUSED_NORM_PROLOGUE");
    return v && v[0] == '0';
  }();
  if (off) return CEK_ERR_UNSUPPORTED;
  p.x = hidden;
  p.residual = residual;
  p.gamma = gamma;
  p.norm = 1;
  p.eps = eps;
  int s = gemv_bulk_launch(p, dtype, dtype, w_fmt, scale_kind, st);
  if (s != CEK_OK) return s;
  const int nvec = p.M * p.K / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(148, (nvec + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = cek_host::pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, residual_update_kernel<T>, static_cast<const T*>(hidden), static_cast<T*>(residual),
                         nvec) != cudaSuccess)
    return CEK_ERR_LAUNCH;
  return cek_host::launch_status();
}

}  // namespace cek

namespace {
int check_norm_args(const void* hidden, const void* residual, int64_t rows, int64_t K, int dtype) {
  if (rows < 0 || K <= 0 || K % 8 != 0 || K > 16384) return CEK_ERR_INVALID_ARG;
  if (dtype != CEK_F16 && dtype != CEK_BF16) return CEK_ERR_INVALID_ARG;
  if (rows > 0 && (!hidden || !residual)) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(hidden) || !cek_host::aligned16(residual)) return CEK_ERR_ALIGNMENT;
  return CEK_OK;
}
}  // namespace

extern "C" int cek_fused_add_rmsnorm(void* hidden, void* residual, const void* weight, int64_t rows,
                                     int64_t K, float eps, int dtype, void* stream) {
  int s = check_norm_args(hidden, residual, rows, K, dtype);
  if (s != CEK_OK) return s;
  if (rows == 0) return CEK_OK;
  if (!weight) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(weight)) return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == CEK_F16)
    return cek::launch_norm<__half, cek::kNormedInPlace>(hidden, residual, weight, nullptr, nullptr, rows, K,
                                                         eps, st);
  return cek::launch_norm<__nv_bfloat16, cek::kNormedInPlace>(hidden, residual, weight, nullptr, nullptr, rows,
                                                                K, eps, st);
}

// Workspace.  With at least cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K)
// bytes the stats kernel writes the normalised rows (M x K, I/O dtype, an
// L2-resident scratch) and the GEMV runs its plain operand path on them.
// With only the 256-byte inverse-RMS block the stats kernel writes the
// per-row inverse RMS and the GEMV forms the normalised operand inside its
// loads (slower: every warp redoes the scaling).
static int64_t inv_rms_bytes(int64_t M) { return ((M * (int64_t)sizeof(float) + 255) / 256) * 256; }
static int64_t normed_bytes(int64_t M, int64_t K) { return ((M * K * 2 + 255) / 256) * 256; }

extern "C" int64_t cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(int64_t M, int64_t K) {
  if (M <= 0 || M > 16 || K <= 0 || K > 16384) return 0;
  return normed_bytes(M, K);
}

extern "C" int cek_fused_add_rmsnorm_gemv_fp8(const void* hidden, void* residual,
                                              const void* norm_weight, float eps, const void* w,
                                              const void* scale, void* y, void* workspace,
                                              int64_t workspace_bytes, int64_t M, int64_t N,
                                              int64_t K, int dtype, int w_fmt, int scale_kind,
                                              unsigned flags, void* stream) {
  int s = check_norm_args(hidden, residual, M, K, dtype);
  if (s != CEK_OK) return s;
  if (M > 16 || N < 0 || workspace_bytes < 0) return CEK_ERR_INVALID_ARG;
  if (w_fmt != CEK_E4M3 && w_fmt != CEK_E5M2) return CEK_ERR_INVALID_ARG;
  if (scale_kind < CEK_SCALE_PERN_F16 || scale_kind > CEK_SCALE_PERT_F32) return CEK_ERR_INVALID_ARG;
  if (flags & ~(unsigned)(CEK_GEMV_EARLY_WEIGHTS | CEK_GEMV_GELU_MUL_OUTPUT)) return CEK_ERR_INVALID_ARG;
  if (M == 0) return CEK_OK;
  if (!norm_weight || !w || !scale || !workspace || (N > 0 && !y)) return CEK_ERR_INVALID_ARG;
  const bool gelu_out = (flags & CEK_GEMV_GELU_MUL_OUTPUT) != 0;
  // the gated output is formed by the bulk GEMV, which reads staged rows
  if (gelu_out && (workspace_bytes < normed_bytes(M, K) || M > 16 || K % 64 != 0)) return CEK_ERR_UNSUPPORTED;
  if (workspace_bytes < inv_rms_bytes(M)) return CEK_ERR_INVALID_ARG;
  if (!cek_host::aligned16(norm_weight) || !cek_host::aligned16(w) || !cek_host::aligned16(workspace))
    return CEK_ERR_ALIGNMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // On chip up to K = 4096: at K = 8192 (the 70B chain, M = 1) the two-kernel
  // path measured faster inside the decode step (144.9 against 149.0 us per
  // layer), although a lone fused call is faster on chip.
  if (N > 0 && K % 64 == 0 && K <= 4096) {
    cek::GemvParams q = {};
    q.w = static_cast<const uint8_t*>(w); q.scale = scale; q.y = y;
    q.M = (int)M; q.N = (int)N; q.K = (int)K;
    q.early_weights = 1;  // nothing in front of the GEMV writes W
    q.y_gelu = gelu_out ? 1 : 0;
    s = dtype == CEK_F16
            ? cek::fused_norm_gemv_onchip<__half>(hidden, residual, norm_weight, eps, q, dtype, w_fmt, scale_kind, st)
            : cek::fused_norm_gemv_onchip<__nv_bfloat16>(hidden, residual, norm_weight, eps, q, dtype, w_fmt,
                                                         scale_kind, st);
    if (s != CEK_ERR_UNSUPPORTED) return s;
  }
  const bool staged = workspace_bytes >= normed_bytes(M, K);
  float* inv = static_cast<float*>(workspace);
  // The stats kernel only reads `hidden`; the const_cast never leads to a write.
  void* h = const_cast<void*>(hidden);
  if (staged)
    s = dtype == CEK_F16
            ? cek::launch_norm<__half, cek::kNormedOut>(h, residual, norm_weight, nullptr, workspace, M, K, eps, st)
            : cek::launch_norm<__nv_bfloat16, cek::kNormedOut>(h, residual, norm_weight, nullptr, workspace, M, K,
                                                               eps, st);
  else
    s = dtype == CEK_F16
            ? cek::launch_norm<__half, cek::kInvRmsOnly>(h, residual, nullptr, inv, nullptr, M, K, eps, st)
            : cek::launch_norm<__nv_bfloat16, cek::kInvRmsOnly>(h, residual, nullptr, inv, nullptr, M, K, eps, st);
  if (s != CEK_OK || N == 0) return s;
  cek::GemvParams p = {};
  p.w = static_cast<const uint8_t*>(w); p.scale = scale; p.y = y;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  // The stats kernel never writes W: the GEMV may always prefetch it.
  p.early_weights = 1;
  p.y_gelu = gelu_out ? 1 : 0;
  if (staged) {
    p.x = workspace;
    return cek::gemv_launch(p, dtype, dtype, w_fmt, scale_kind, false, st);
  }
  p.x = nullptr;
  p.residual = residual; p.gamma = norm_weight; p.inv_rms = inv;
  return cek::gemv_launch(p, dtype, dtype, w_fmt, scale_kind, true, st);
}

// ---- no-allocation variant ---------------------------------------------------
// The fused op's inverse-RMS scratch as a fixed device array, sized like the
// op's workspace for CEK_NOALLOC_MAX_ROWS rows (256 bytes).  Host code must
// not hand `g_noalloc_inv_rms` itself to a kernel: on the host that name is a
// shadow variable, not device memory.  It passes the device address that
// cudaGetSymbolAddress returns in the calling thread's current CUDA context.
// That address belongs to the context it was looked up in (a module is loaded
// once per context), so the cache holds one entry per device, tagged with the
// unique ID of the context (cuCtxGetId, reached through the runtime's driver
// entry-point query so the library needs no libcuda link): a call from another
// context on the same device, or from the context the runtime re-creates after
// cudaDeviceReset, looks the address up again.
constexpr int kNoallocFloats =
    int((CEK_NOALLOC_MAX_ROWS * sizeof(float) + 255) / 256 * 256 / sizeof(float));
static __device__ __align__(256) float g_noalloc_inv_rms[kNoallocFloats];

namespace {
constexpr int kMaxDevices = 64;
struct NoallocEntry { unsigned long long ctx_id; float* addr; };
std::mutex g_noalloc_mu;
NoallocEntry g_noalloc[kMaxDevices] = {};

// The current context's unique ID (0 when it cannot be read: the cache is then
// bypassed and the address looked up on every call).
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static const std::pair<GetCurrent, GetId> fns = [] {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa = cudaDriverEntryPointSymbolNotFound, qb = qa;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 12000, cudaEnableDefault, &qa) != cudaSuccess ||
        qa != cudaDriverEntryPointSuccess)
      a = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) != cudaSuccess ||
        qb != cudaDriverEntryPointSuccess)
      b = nullptr;
    return std::make_pair(reinterpret_cast<GetCurrent>(a), reinterpret_cast<GetId>(b));
  }();
  if (!fns.first || !fns.second) return 0;
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (fns.first(&ctx) != 0 || !ctx || fns.second(ctx, &id) != 0) return 0;
  return id;
}

int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CEK_ERR_LAUNCH;
  if (dev < 0 || dev >= kMaxDevices) return CEK_ERR_UNSUPPORTED;
  // cudaGetSymbolAddress makes the runtime bind (or create) the device's
  // context first, so the context ID is read after it on a miss
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocEntry& e = g_noalloc[dev];
  if (id == 0 || e.ctx_id != id || !e.addr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_inv_rms) != cudaSuccess || !p) return CEK_ERR_LAUNCH;
    e.addr = static_cast<float*>(p);
    e.ctx_id = current_context_id();
  }
  *out = e.addr;
  return CEK_OK;
}
}  // namespace

extern "C" int cek_fused_add_rmsnorm_gemv_fp8_noalloc(const void* hidden, void* residual,
                                                      const void* norm_weight, float eps,
                                                      const void* w, const void* scale, void* y,
                                                      int64_t M, int64_t N, int64_t K, int dtype,
                                                      int w_fmt, int scale_kind, unsigned flags,
                                                      void* stream) {
  if (M > CEK_NOALLOC_MAX_ROWS) return CEK_ERR_SCRATCH_LIMIT;
  if (M < 0) return CEK_ERR_INVALID_ARG;
  if (M == 0) return CEK_OK;
  float* scratch = nullptr;
  const int s = noalloc_scratch(&scratch);
  if (s != CEK_OK) return s;
  return cek_fused_add_rmsnorm_gemv_fp8(hidden, residual, norm_weight, eps, w, scale, y, scratch,
                                        int64_t(sizeof(g_noalloc_inv_rms)), M, N, K, dtype, w_fmt,
                                        scale_kind, flags, stream);
}
