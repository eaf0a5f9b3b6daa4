// Bulk asynchronous copies (the TMA engine's 1D form, cp.async.bulk) into shared memory with
// mbarrier completion, and bounded waits.  No multicast anywhere: every copy reads this GPU's
// own global memory into the issuing CTA's shared memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "g4_common.cuh"

namespace g4 {

// Device status word of this translation unit: bit 0 = a bounded wait gave up; bit 1 = a CTA
// returned after a wait gave up while its own copies (or tensor-core operations) could still be in
// flight, so shared or tensor memory that a later CTA owns may have been written.  Each .cu file
// gets its own copy (no relocatable device code); G4_STATUS_READER(name) defines the host
// reader that g4_device_status() calls for it.
static __device__ unsigned int g_dev_status = 0;
constexpr unsigned kStatusTimeout = 1u;
constexpr unsigned kStatusInflight = 2u;
// Every device-side wait gives up after this long (ns on %globaltimer).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }


__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes barrier initialisation visible to the async proxy before any copy targets it.
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// 1D bulk copy global -> this CTA's shared memory; dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Wait for phase `parity` of the barrier, giving up after `limit_ns`.  Returns true on success.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}
// CTA-uniform wait: every thread polls; if any gave up, the status word is flagged and all threads
// learn it together (so none is left at a later __syncthreads).  Returns true when all succeeded.
// On failure thread 0 waits once more (bounded) for the CTA's copies still in flight before the
// CTA returns, so no copy lands in shared memory that a later CTA owns.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  const int any_fail = __syncthreads_or(!ok);
  if (any_fail) {
    if (threadIdx.x == 0) {
      atomicOr(&g_dev_status, kStatusTimeout);
      if (!mbar_wait(bar, parity)) atomicOr(&g_dev_status, kStatusInflight);
    }
    __syncthreads();
  }
  return !any_fail;
}
// 2D tiled tensor load (TMA) global -> this CTA's shared memory, completion on an mbarrier.  The
// innermost coordinate x (in elements) times the element size must be a multiple of 16 bytes.
// No cluster multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before its later
// async-proxy (bulk copy) writes into the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace g4

#define G4_STATUS_READER(name)                                                              \
  namespace g4 {                                                                            \
  unsigned status_read_##name(bool reset) {                                                 \
    unsigned v = 0;                                                                         \
    cudaMemcpyFromSymbol(&v, g_dev_status, sizeof v);                                       \
    if (reset) { const unsigned z = 0; cudaMemcpyToSymbol(g_dev_status, &z, sizeof z); }   \
    return v;                                                                               \
  }                                                                                         \
  }
