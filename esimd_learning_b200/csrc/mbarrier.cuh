// mbarrier.cuh — shared-memory mbarrier and 1-D bulk-copy helpers (sm_90+
// PTX) for the producer/consumer kernels.  Every wait is bounded by the
// caller's poll limit.
#pragma once
#include "common.cuh"

namespace cek {
namespace mbar {

CEK_DEVICE uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CEK_DEVICE void init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
CEK_DEVICE void fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

CEK_DEVICE bool try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete; false after `polls`
// unsuccessful polls.
CEK_DEVICE bool wait(uint32_t bar, uint32_t parity, uint32_t polls) {
  for (uint32_t i = 0; i < polls; ++i)
    if (try_wait(bar, parity)) return true;
  return false;
}
CEK_DEVICE void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
CEK_DEVICE void arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  dst, src 16-byte aligned; bytes a multiple of 16.  No
// multicast.
CEK_DEVICE void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
CEK_DEVICE uint4 lds16(uint32_t a) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
  return r;
}

}  // namespace mbar
}  // namespace cek
