// common.cuh — shared device helpers for the sm_100a FP8 custom-op kernels.
//
// FP8 -> 16-bit conversion.  The reference dequantises with integer bit
// tricks and flushes FP8 subnormals to zero (csrc/xpu/esimd_kernels/
// fp8_GEMV_v2.h:12-38).  Here every conversion is exact (subnormals kept),
// which is what the reference tests' oracle `weight_fp8.to(torch.float16)`
// computes (tests/test_gemv_fp8.py:31-32); both FP8 formats embed exactly in
// fp16 and in bf16, so no rounding happens on the weight path.
#pragma once
#include <atomic>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cstdlib>

#include "../../include/cek.h"

#define CEK_DEVICE __device__ __forceinline__

namespace cek {

// ---- 16-byte global loads ---------------------------------------------------
// Weights are read exactly once per call: bypass L1 so the L1/shared carve-out
// stays with the activation tiles.
CEK_DEVICE uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
CEK_DEVICE uint4 ldg_nc(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- FP8 pair -> packed 16-bit pair -------------------------------------------
// `pair` holds two FP8 codes in its low 16 bits (byte 0 -> low half of the
// result, byte 1 -> high half), matching the mma.sync fragment convention that
// the lower 16 bits carry the lower k index.
template <int FMT, int HI = 0>
CEK_DEVICE uint32_t fp8x2_to_f16x2(uint32_t pair) {
  // HI = 1 converts bytes 2 and 3 of `pair` instead of bytes 0 and 1.
  uint32_t r;
  if constexpr (FMT == CEK_E4M3) {
    if constexpr (HI)
      asm("{ .reg .b16 lo, hi; mov.b32 {lo, hi}, %1; cvt.rn.f16x2.e4m3x2 %0, hi; }" : "=r"(r) : "r"(pair));
    else
      asm("{ .reg .b16 lo; mov.b32 {lo, _}, %1; cvt.rn.f16x2.e4m3x2 %0, lo; }" : "=r"(r) : "r"(pair));
  } else {
    // e5m2 is the top byte of an fp16: place each byte in the high half of its lane.
    r = __byte_perm(pair, 0u, HI ? 0x3424 : 0x1404);
  }
  return r;
}

// Exact FP8 -> bf16 for a pair.  The FP8 exponent/mantissa field is placed at
// the bottom of the bf16 exponent field, which makes the bf16 value equal to
// the FP8 value times 2^-(127 - bias); one exact bf16x2 multiply by
// 2^(127 - bias) restores it.  FP8 subnormals land on bf16 subnormals, which
// the multiply handles exactly (bf16 arithmetic on sm_90+ keeps subnormals).
template <int FMT, int HI = 0>
CEK_DEVICE uint32_t fp8x2_to_bf16x2(uint32_t pair) {
  uint32_t v = __byte_perm(pair, 0u, HI ? 0x4342 : 0x4140);  // [b0, 0, b1, 0] (HI: bytes 2, 3)
  uint32_t r;
  if constexpr (FMT == CEK_E4M3) {
    r = ((v & 0x007F007Fu) << 4) | ((v & 0x00800080u) << 8);
    const uint32_t k2p120 = 0x7B807B80u;  // bf16x2 (2^120, 2^120)
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(r), "r"(k2p120));
  } else {
    r = ((v & 0x007F007Fu) << 5) | ((v & 0x00800080u) << 8);
    const uint32_t k2p112 = 0x77807780u;  // bf16x2 (2^112, 2^112)
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(r), "r"(k2p112));
  }
  return r;
}

// ---- scalar conversions ------------------------------------------------------
template <typename T> CEK_DEVICE float to_f32(T v);
template <> CEK_DEVICE float to_f32<__half>(__half v) { return __half2float(v); }
template <> CEK_DEVICE float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> CEK_DEVICE T from_f32(float v);
template <> CEK_DEVICE __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> CEK_DEVICE __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Packed pair <-> two floats (low half first).
template <typename T> CEK_DEVICE float2 unpack2(uint32_t u);
template <> CEK_DEVICE float2 unpack2<__half>(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}
template <> CEK_DEVICE float2 unpack2<__nv_bfloat16>(uint32_t u) {
  __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(h);
}
template <typename T> CEK_DEVICE uint32_t pack2(float a, float b);
template <> CEK_DEVICE uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> CEK_DEVICE uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---- GeLU(tanh)-and-mul ------------------------------------------------------
// gelu_tanh(g) = 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))), in fp32 with
// every rounding step pinned (no contraction choices left to the compiler),
// so the standalone op and the GEMV prologue that forms the same product
// produce identical bits.
CEK_DEVICE float gelu_tanh(float g) {
  const float kAlpha = 0.7978845608028654f;  // sqrt(2/pi)
  const float kBeta = 0.044715f;
  const float inner = __fmul_rn(kAlpha, __fmaf_rn(__fmul_rn(kBeta, __fmul_rn(g, g)), g, g));
  return __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.f, tanhf(inner)));
}
// io(gelu_tanh(g) * u) for a packed pair of 16-bit values.
template <typename T>
CEK_DEVICE uint32_t gelu_mul2(uint32_t g2, uint32_t u2) {
  const float2 g = unpack2<T>(g2), u = unpack2<T>(u2);
  return pack2<T>(__fmul_rn(gelu_tanh(g.x), u.x), __fmul_rn(gelu_tanh(g.y), u.y));
}

template <typename T>
CEK_DEVICE T gelu_mul1(T g, T u) {
  return from_f32<T>(__fmul_rn(gelu_tanh(to_f32<T>(g)), to_f32<T>(u)));
}

// ---- warp / block reductions -------------------------------------------------
CEK_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
CEK_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- programmatic dependent launch (PDL) ----------------------------------------
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start while its predecessor on the stream is still running; it must call
// pdl_wait() before touching anything the predecessor writes.  Without the
// attribute both instructions are no-ops.
CEK_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CEK_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace cek

// Host helpers shared by the launch files.
namespace cek_host {
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// Programmatic dependent launch is on unless CEK_DISABLE_PDL=1 is set.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("CEK_DISABLE_PDL");
    return !(v && v[0] == '1');
  }();
  return on;
}
// Per-device host caches (SM count, configured shared-memory size).  Slots
// are atomics, so host threads launching concurrently see either the old or
// the new value; both writers store the same value, and the cached work
// (an attribute query, cudaFuncSetAttribute) is idempotent.  Ordinals at or
// above kMaxCachedDevices are not cached: the work is redone on every call.
constexpr int kMaxCachedDevices = 64;
struct DeviceSlots {
  std::atomic<int> v[kMaxCachedDevices] = {};
  std::atomic<int>* at(int dev) { return dev >= 0 && dev < kMaxCachedDevices ? &v[dev] : nullptr; }
};
// SM count of the current device, cached per device (launch planning runs
// on every call; the attribute query is host time on the hot path).
inline int sm_count() {
  static DeviceSlots cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>* c = cache.at(dev);
  int v = c ? c->load(std::memory_order_relaxed) : 0;
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    if (c) c->store(v, std::memory_order_relaxed);
  }
  return v;
}
// Raise a kernel's dynamic shared-memory limit to `bytes` once per device.
template <typename Kern>
inline bool ensure_smem_attr(DeviceSlots& slots, Kern kern, int bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>* c = slots.at(dev);
  if (c && c->load(std::memory_order_relaxed) >= bytes) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (c) c->store(bytes, std::memory_order_relaxed);
  return true;
}
// Launch with programmatic stream serialization (unless CEK_DISABLE_PDL=1):
// the kernel may start while the previous kernel on the stream drains; it
// must execute griddepcontrol.wait before touching anything that kernel
// writes.
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...) == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CEK_OK : CEK_ERR_LAUNCH;
}
}  // namespace cek_host
