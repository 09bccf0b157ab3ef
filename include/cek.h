/*
 * cek.h — C ABI of the B200 (sm_100a) FP8 custom-op library `libcek_b200.so`.
 *
 * Every entry point takes plain device pointers, sizes and enums, enqueues its
 * kernels on the CUDA stream passed as `stream` (a `cudaStream_t` cast to
 * `void*`; NULL means the legacy default stream), never synchronises with the
 * host, and returns a `cek_status` (0 = success).  No torch type crosses this
 * boundary; the thin torch-library registration (csrc/torch_extension*.cc)
 * turns a non-zero status into a Python RuntimeError via TORCH_CHECK.
 *
 * The reference (Intel ESIMD/SYCL, "custom-esimd-kernels-vllm") has no C ABI:
 * its launch layer is a set of C++ functions taking at::Tensor.  Each entry
 * point below names the reference function whose work it replaces, so a
 * maintainer can map the reference's launch layer onto this library one to
 * one.  All tensors are row-major and contiguous.
 */
#ifndef CEK_H_
#define CEK_H_

#include <stdint.h>

#if defined(__GNUC__)
#define CEK_API __attribute__((visibility("default")))
#else
#define CEK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
typedef enum {
  CEK_OK = 0,
  CEK_ERR_INVALID_ARG = 1,  /* bad size, null pointer, unknown enum value     */
  CEK_ERR_UNSUPPORTED = 2,  /* valid arguments this build does not implement  */
  CEK_ERR_ALIGNMENT = 3,    /* pointer or row pitch not 16-byte aligned       */
  CEK_ERR_LAUNCH = 4,       /* cudaGetLastError() reported a launch failure   */
  CEK_ERR_TIMEOUT = 5,      /* a bounded device-side wait ran out             */
  CEK_ERR_SCRATCH_LIMIT = 6, /* size above the fixed scratch of a no-allocation entry point */
} cek_status;

/* ---- element-type enums --------------------------------------------------- */
typedef enum { CEK_F16 = 0, CEK_BF16 = 1 } cek_io_dtype;
/* Same numbering as the reference's fp8_mode (esimd_kernel.sycl:14-16). */
typedef enum { CEK_E4M3 = 0, CEK_E5M2 = 1 } cek_fp8_format;
typedef enum {
  CEK_SCALE_PERN_F16 = 0, /* fp16[N]: the reference's per-N scale            */
  CEK_SCALE_PERN_F32 = 1, /* fp32[N]: per-output-channel scale               */
  CEK_SCALE_PERT_F32 = 2, /* fp32 scalar on the device: per-tensor scale     */
} cek_scale_kind;

/* Human-readable name of a status code (static storage, never NULL). */
CEK_API const char* cek_status_string(int status);

/* Library version string, e.g. "cek_b200 0.1 sm_100a". */
CEK_API const char* cek_version(void);

/* ---- FP8-weight GEMV / small-M GEMM --------------------------------------
 * y[m, n] = OutT( sum_k f32(x[m, k]) * f32(deq(w[n, k])) * scale(n) )
 * x: [M, K] x_dtype; w: [N, K] fp8 (w_fmt); y: [M, N] y_dtype.
 * scale(n) = scale[n] (per-N kinds) or scale[0] (per-tensor), read on device.
 * Any M >= 1; K % 16 == 0; x and w 16-byte aligned.  No scratch memory.
 *
 * The kernel is launched with programmatic dependent launch (PDL): it may
 * start while the previous kernel on `stream` finishes.  By default every
 * global read waits for that kernel.  flags |= CEK_GEMV_EARLY_WEIGHTS lets
 * the weight stream start before the wait (hiding launch and DRAM latency);
 * the caller then guarantees that the kernel launched immediately before on
 * `stream` does not write w.
 * Replaces: GEMV_fp8_pern_host  (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:171),
 *           GEMV_fp8_pert_host  (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:414),
 *           GEMM_fp8_pert_dispatch, M <= 64 (csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:4017). */
#define CEK_GEMV_EARLY_WEIGHTS 1u
/* flags |= CEK_GEMV_GELU_MUL_OUTPUT: gated output for the decode MLP's
 * gate_up projection with GeLU-and-mul fused into its epilogue.  w holds 2N
 * rows, the gate rows [0, N) then the up rows [N, 2N) (vLLM's merged
 * gate_up layout); a per-N scale has 2N entries.  y is [M, N]:
 *   y[m, n] = io( gelu_tanh(f32 g) * f32 u ),  g = io(GEMV row n),
 *   u = io(GEMV row N + n),
 * i.e. bit for bit the plain GEMV into [M, 2N] followed by cek_gelu_and_mul,
 * in one launch and without the [M, 2N] round trip.  Supported for M <= 16,
 * K % 64 == 0 and x_dtype == y_dtype; otherwise CEK_ERR_UNSUPPORTED and nothing runs.  New: the
 * reference has no GeLU op. */
#define CEK_GEMV_GELU_MUL_OUTPUT 2u
CEK_API int cek_gemv_fp8(const void* x, const void* w, const void* scale, void* y,
                         int64_t M, int64_t N, int64_t K, int x_dtype, int y_dtype,
                         int w_fmt, int scale_kind, unsigned flags, void* stream);

/* ---- several FP8 GEMVs sharing one activation, one launch ---------------
 * For m < count: ys[m][M, Ns[m]] = GEMV(x, ws[m] [Ns[m], K], scales[m]) as
 * cek_gemv_fp8 (one scale kind and FP8 format for all).  count <= 4; the
 * pointer arrays are HOST arrays of device pointers.  Saves the launch and
 * ramp of each extra matrix (e.g. gate + up, qkvz + ba).
 * Replaces: GEMV_fp8_pern_fused_host (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:262),
 *           GEMV_fp8_pert_fused_host (csrc/xpu/esimd_kernels/fp8_GEMV_v2.h:505). */
CEK_API int cek_gemv_fp8_multi(const void* x, const void* const* ws, const void* const* scales,
                               void* const* ys, const int64_t* Ns, int count, int64_t M, int64_t K,
                               int x_dtype, int y_dtype, int w_fmt, int scale_kind, unsigned flags,
                               void* stream);

/* ---- residual add + RMSNorm (batched, in place) ---------------------------
 * residual[r, :] = fp16(hidden[r, :] + residual[r, :])
 * hidden[r, :]   = fp16(f32(residual[r, :]) * rsqrt(mean((h + r)^2) + eps) * weight)
 * weight is the Gemma-style pre-shifted (w + 1) vector.  rows >= 0, K % 8 == 0,
 * K <= 16384.  Replaces: fused_add_rms_norm_batched_host
 * (csrc/xpu/esimd_kernels/fused_add_rms_norm_batched.h:66). */
CEK_API int cek_fused_add_rmsnorm(void* hidden, void* residual, const void* weight,
                          int64_t rows, int64_t K, float eps, int dtype,
                          void* stream);

/* ---- residual add + RMSNorm fused into an FP8 GEMV ------------------------
 * residual = io(hidden + residual)  (in place; hidden is not written)
 * xn       = io(f32(residual) * inv_rms[m] * weight)
 * y        = GEMV(xn, w, scale)  as cek_gemv_fp8.
 * Where x [M, K] fits in the bulk GEMV's shared memory beside its weight
 * ring and K <= 4096 (M <= 2 at K = 4096; e4m3 weights, K % 64 == 0)
 * the GEMV itself forms xn on chip: every CTA reads hidden and residual,
 * reduces the inverse RMS and stages xn, then a small kernel launched
 * behind it (once all CTAs have read the residual) writes the residual.
 * The workspace is not touched there.  Otherwise two launches chained by
 * programmatic dependent launch: a per-row stats kernel (residual update
 * and normalisation) and the GEMV, which streams w while the stats kernel
 * runs.
 * workspace (contents ignored; required either way):
 *   >= cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(M, K) bytes: the stats
 *      kernel writes xn there (M x K, L2-resident) and the GEMV reads it;
 *   >= 256 bytes only: the stats kernel writes the per-row inverse RMS and
 *      the GEMV forms xn inside its operand loads (slower).
 * flags: CEK_GEMV_EARLY_WEIGHTS is accepted and implied (the weight stream
 * always starts early here: the stats kernel never writes w);
 * CEK_GEMV_GELU_MUL_OUTPUT makes the projection the gated gate_up one of
 * cek_gemv_fp8 (w [2N, K], y [M, N]); it needs the full workspace, M <= 16 and
 * K % 64 == 0, else CEK_ERR_UNSUPPORTED before anything runs.
 * M <= 16, K % 8 == 0, K <= 16384.  No reference counterpart: the reference
 * runs fused_add_rms_norm_batched_host and GEMV_fp8_pern_host as two ops. */
CEK_API int64_t cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(int64_t M, int64_t K);
CEK_API int cek_fused_add_rmsnorm_gemv_fp8(const void* hidden, void* residual,
                                           const void* norm_weight, float eps,
                                           const void* w, const void* scale, void* y,
                                           void* workspace, int64_t workspace_bytes,
                                           int64_t M, int64_t N, int64_t K, int dtype,
                                           int w_fmt, int scale_kind, unsigned flags,
                                           void* stream);

/* ---- the same fused op, with no allocation at all -------------------------
 * For callers that cannot allocate device memory where they call this op:
 * code running where cudaMalloc is forbidden or unavailable (a plugin's
 * enqueue callback inside another runtime), a process whose GPU memory is
 * handed out by its own pool at start-up, or a serving loop that must not
 * touch an allocator per request.  They pass inputs and outputs only.
 *
 * Computes what cek_fused_add_rmsnorm_gemv_fp8 computes when that entry point
 * is given only the small inverse-RMS workspace: the same residual bits, and
 * a projection within the GEMV tolerance of the full-workspace result (the
 * normalised operand is formed in a different place, so it is not
 * bit-identical).  CEK_GEMV_GELU_MUL_OUTPUT is refused with
 * CEK_ERR_UNSUPPORTED: the gated output needs the full workspace.
 * Its per-row inverse-RMS scratch is a fixed device array inside
 * libcek_b200.so, sized for CEK_NOALLOC_MAX_ROWS rows (256 bytes); every GPU
 * that loads the library holds it until the process exits.
 * M > CEK_NOALLOC_MAX_ROWS returns CEK_ERR_SCRATCH_LIMIT.  The array needs no
 * clearing (each call writes every row it later reads), but all calls share
 * it: calls that overlap on the GPU (different streams, or different host
 * threads on one device) race.
 * The array's device address is looked up (cudaGetSymbolAddress) by the first
 * call in each CUDA context, with that context current, and cached per device
 * under the context's unique ID; a call from a different context on the same
 * device (a non-primary context, or the one re-created after
 * cudaDeviceReset) looks it up again.  Make the first call in a context
 * before any stream capture.  No counterpart in the reference. */
#define CEK_NOALLOC_MAX_ROWS 16
CEK_API int cek_fused_add_rmsnorm_gemv_fp8_noalloc(const void* hidden, void* residual,
                                                   const void* norm_weight, float eps,
                                                   const void* w, const void* scale, void* y,
                                                   int64_t M, int64_t N, int64_t K, int dtype,
                                                   int w_fmt, int scale_kind, unsigned flags,
                                                   void* stream);

/* ---- GeLU(tanh)-and-mul ----------------------------------------------------
 * out[m, j] = gelu_tanh(x[m, j]) * x[m, d + j];  x: [M, 2d], out: [M, d].
 * Any d >= 0 (d % 8 == 0: 16-byte vectors, x and out 16-byte aligned;
 * otherwise element by element).  No reference counterpart (vLLM's
 * gelu_tanh_and_mul layout). */
CEK_API int cek_gelu_and_mul(const void* x, void* out, int64_t M, int64_t d, int dtype,
                     void* stream);

/* ---- per-head RMSNorm on q and k, then rotary embedding (in place) --------
 * qkv: [M, (Hq + 2*Hkv) * D]; q heads first, then k heads, then v (untouched).
 * q_weight, k_weight: [D] norm weights (plain multiply, not shifted).
 * positions: int64 [M]; cos_sin_cache: fp32 [max_pos, D] with cos in the first
 * D/2 columns and sin in the last D/2 (vLLM layout).  is_neox selects the
 * rotate-half (1) or interleaved-pair (0) rotary convention.  D in {64,128,256}.
 * No reference counterpart. */
CEK_API int cek_qkv_norm_rope(void* qkv, const int64_t* positions, const void* q_weight,
                      const void* k_weight, const float* cos_sin_cache,
                      int64_t M, int64_t num_q_heads, int64_t num_kv_heads,
                      int64_t head_dim, int64_t max_position, float eps,
                      int is_neox, int dtype, void* stream);

/* ---- per-token dynamic e4m3 quantisation ----------------------------------
 * s[m] = max(amax(|a[m, :]|), 1e-12) / 448;  aq[m, k] = e4m3_rn(clamp(a / s[m])).
 * a: [M, K] fp16/bf16; aq: [M, K] e4m3; s: fp32 [M].  K % 8 == 0, K <= 16384.
 * No reference counterpart (the reference GEMM takes fp16 activations). */
CEK_API int cek_quant_fp8_per_token(const void* a, void* aq, float* a_scale, int64_t M,
                            int64_t K, int dtype, void* stream);

/* ---- tensor parallel: row-parallel FP8 GEMV fused with its all-reduce -----
 * out[m, n] = sum over the `world` ranks of GEMV(x_r, w_r, scale)[m, n],
 * every rank getting the same bits.  Each rank owns a comm region of
 * cek_tp_comm_bytes(slot_elems, world) bytes from cek_comm_alloc (zeroed);
 * ranks exchange its CUDA IPC handle (cek_ipc_get_handle / cek_ipc_open_handle)
 * and pass `peer_comm`, a DEVICE array of `world` 64-bit addresses of every
 * rank's region as mapped in this process (own region at index rank).
 * The GEMV's epilogue pushes its tiles into every rank's region over NVLink
 * while later tiles are still computing; a second small kernel raises this
 * rank's ready flag on every rank, waits for all ranks' flags (bounded), adds
 * the slots in rank order and writes `out`.
 * M * N <= slot_elems; K % 16 == 0; one call at a time per region.
 * Bounded waits that run out set bit 0 of the region's error word
 * (cek_comm_errors).  The word is sticky: after a timeout the ranks' epochs
 * may disagree, so the call's output and every later one are suspect until
 * the regions are reset.  Recovery: stop launching on every rank, agree on the
 * host (a store or a barrier), then cek_comm_reset every rank's region (zeroes
 * epoch, flags, error word and slots; synchronising) before the next call.
 * No reference counterpart: the reference is single-GPU.
 * cek_comm_alloc / cek_comm_free / the IPC calls are set-up calls (they
 * allocate or map memory and synchronise); the GEMV call does neither. */
#define CEK_IPC_HANDLE_BYTES 64
CEK_API int64_t cek_tp_comm_bytes(int64_t slot_elems, int world);
CEK_API int cek_comm_alloc(int64_t bytes, void** ptr);
CEK_API int cek_comm_free(void* ptr);
CEK_API int cek_ipc_get_handle(void* ptr, void* handle);
CEK_API int cek_ipc_open_handle(const void* handle, void** ptr);
CEK_API int cek_ipc_close_handle(void* ptr);
CEK_API int cek_comm_errors(void* my_comm, uint32_t* out);
CEK_API int cek_comm_reset(void* my_comm, int64_t bytes);
/* ---- tensor parallel: column-parallel FP8 GEMV fused with its all-gather --
 * This rank holds rows [row0, row0 + N) of the weight (and their scales) and
 * computes those rows of y [M, n_full] = x @ deq(W)^T * scale; the epilogue
 * stores them over NVLink into every rank's copy of y, which sits at byte
 * offset y_off of the data area (CEK_COMM_SYNC_BYTES into the region) of
 * each rank's comm region (comm_bytes long, set up as for the all-reduce).
 * No barrier inside: after the step's all-gather GEMVs, cek_comm_barrier on
 * every rank makes all ranks' rows visible everywhere.  A y buffer must not
 * be written by the next call before every rank has finished reading it
 * (alternate two buffers by step parity).  Replaces the NCCL all-gather that
 * follows a column-parallel GEMV; no reference counterpart (single-GPU). */
#define CEK_COMM_SYNC_BYTES 4096
CEK_API int cek_gemv_fp8_allgather(const void* x, const void* w, const void* scale, int64_t M, int64_t N,
                                   int64_t K, int64_t row0, int64_t n_full, int64_t y_off, int dtype,
                                   int w_fmt, int scale_kind, const uint64_t* peer_comm, void* my_comm,
                                   int64_t comm_bytes, int rank, int world, unsigned flags, void* stream);
/* Barrier over the comm regions of all ranks, on the stream after the
 * pushes it covers (one bounded wait; a timeout sets the error word). */
CEK_API int cek_comm_barrier(const uint64_t* peer_comm, void* my_comm, int rank, int world, void* stream);
CEK_API int cek_gemv_fp8_allreduce(const void* x, const void* w, const void* scale, void* out,
                                   int64_t M, int64_t N, int64_t K, int dtype, int w_fmt,
                                   int scale_kind, const uint64_t* peer_comm, void* my_comm,
                                   int64_t slot_elems, int rank, int world, unsigned flags,
                                   void* stream);

/* ---- FP8 x FP8 GEMM, per-token x per-channel scales (tcgen05) -------------
 * y[m, n] = OutT( (sum_k deq(aq[m, k]) * deq(bq[n, k])) * a_scale[m] * b_scale[n] )
 * aq: [M, K] e4m3 (e.g. from cek_quant_fp8_per_token); bq: [N, K] e4m3;
 * a_scale fp32 [M]; b_scale fp32 [N]; y: [M, N] y_dtype.
 * K % 128 == 0, N % 16 == 0, any M; aq, bq, y 16-byte aligned.  Persistent
 * tcgen05 kernel (TMA, TMEM accumulators); scratch-free.
 * Replaces the prefill (M > 64) route of GEMM_fp8_pert_dispatch
 * (csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:4043-4048, the scalar
 * weight-stationary kernel), for activations quantised per token. */
CEK_API int cek_gemm_fp8_scaled(const void* aq, const void* bq, const float* a_scale,
                                const float* b_scale, void* y, int64_t M, int64_t N,
                                int64_t K, int y_dtype, void* stream);

/* FP8-weight GEMM with 16-bit activations on the tcgen05 tensor cores:
 *   y[m, n] = T( sum_k x[m, k] * deq(w[n, k]) * scale )
 * Replaces the prefill branch of the reference's esimd_gemm_fp8_pert
 * (csrc/xpu/esimd_kernel_gemm.sycl:23-64 -> GEMM_fp8_pert_dispatch,
 * csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:4043-4048, M > 64).
 * Exact weight conversion (every e4m3/e5m2 value is a 16-bit float of
 * dtype), then kind::f16 tcgen05 MMAs with fp32 accumulation; the scale
 * (fp32 per-tensor scalar, or fp32 per-N) is applied in the epilogue.
 * M <= 256: each weight tile is copied to shared memory as FP8 and
 * converted there by converter warps (workspace untouched; it may be null
 * with workspace_bytes 0).  M > 256: the
 * weight is dequantised once into `workspace`
 * (cek_gemm_fp8w_workspace_bytes(N, K) bytes), then the 16-bit GEMM runs.
 * x, y, T = dtype (CEK_F16 / CEK_BF16), row-major and contiguous.
 * K % 64 == 0 and N % 16 == 0; x, w, y, workspace 16-byte aligned. */
CEK_API int64_t cek_gemm_fp8w_workspace_bytes(int64_t N, int64_t K);
CEK_API int cek_gemm_fp8w(const void* x, const void* w, const void* scale, void* y,
                          void* workspace, int64_t workspace_bytes, int64_t M, int64_t N,
                          int64_t K, int dtype, int w_fmt, int scale_kind, void* stream);
/* Up to this many tokens cek_gemm_fp8w converts the weight in shared memory
 * and never touches the workspace (null with 0 bytes is accepted). */
#define CEK_GEMM_FP8W_INKERNEL_MAX_ROWS 256

/* 1 when a 16-bit-activation FP8-weight product of M tokens should run on
 * cek_gemm_fp8w rather than the GEMV family (cek_gemv_fp8), else 0.  It
 * replaces the fixed decode/prefill cut of the reference's
 * GEMM_fp8_pert_dispatch (csrc/xpu/esimd_kernels/fp8_GEMM_pert.h:4043-4048,
 * M > 64 to the GEMM) with a time estimate from measurements on B200: the
 * GEMV family streams the weight once per 16-token tile, the GEMM once per
 * 128-row block but on no more CTAs than it has 128 x 256 tiles.  Always 0
 * for M <= 16 or shapes the GEMM does not take (K % 64, N % 16), always 1
 * above CEK_GEMM_FP8W_INKERNEL_MAX_ROWS.  Host only, no device work. */
CEK_API int cek_gemm_fp8w_preferred(int64_t M, int64_t N, int64_t K);

/* Number of bounded device waits in the bulk-copy GEMV kernel (the
 * cek_gemv_fp8 path for up to 16 tokens) that gave up since the library was
 * loaded (0 in a healthy run).  Synchronous. */
CEK_API int cek_gemv_fp8_timeouts(uint64_t* count);

/* Number of bounded device waits in cek_gemm_fp8_scaled kernels that gave up
 * since the library was loaded (0 in a healthy run).  Synchronous. */
CEK_API int cek_gemm_fp8_timeouts(uint64_t* count);

#ifdef __cplusplus
}
#endif
#endif /* CEK_H_ */
