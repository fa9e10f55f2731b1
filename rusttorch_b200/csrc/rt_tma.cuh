// rt_tma.cuh — TMA tile loads and mbarrier waits for sm_100a (inline PTX).
//
// Every wait is bounded: mbar_wait gives up after kWaitLimitNs of
// %globaltimer time and returns false, so a kernel whose copy never lands
// records an error and returns instead of spinning.  Every load here fills
// the shared memory of the one CTA that issues it.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace rt {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One bounded probe of the phase.  The suspend-time hint lets the hardware
// park the thread (up to ~10 us) until the phase completes instead of
// spinning, so a waiting warp takes no issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(10000u)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false after
// limit_ns of %globaltimer time.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, unsigned parity,
                                              unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit_ns) return false;
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  return mbar_wait_for(bar, parity, kWaitLimitNs);
}

// A [box] tile of a 3-D tensor map at coordinates (c0 innermost, c1, c2)
// into shared memory; completion is counted on `bar` in bytes.  c0 times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// `bytes` (a multiple of 16) from global `src` to shared `dst` (both 16-byte
// aligned) as one bulk copy, counted on `bar` in bytes.  No multicast: the
// copy fills the issuing CTA's shared memory only.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Host: encodes a tiled tensor map (driver entry point looked up once).
// Returns false if the driver call is unavailable or rejects the layout.
bool encode_tensor_map_f32(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box);

// Host: the device-side flag a kernel sets (to 1) when it gives up a bounded
// wait, for the current device; nullptr if it cannot be resolved.  The
// address is looked up once per device and kept, so the library must not be
// used on a device after that device has been reset.
int* wait_timeout_flag(int device);
// Host: nonzero if a kernel on `device` gave up a bounded wait since the
// last call (the flag is cleared).  Synchronises the device's work first.
int take_wait_timeouts(int device);
// Host: launches a one-thread kernel whose bounded wait runs out (50 ms), to
// exercise the timeout path: the next rtc_synchronize reports it.
cudaError_t launch_bounded_wait_probe(int device, cudaStream_t s);

}  // namespace rt
