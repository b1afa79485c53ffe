// Shared device helpers for the Tokquay paged-attention kernels (sm_100a).
//
// Everything here is plain inline PTX for the TMA bulk-copy engine and
// mbarriers, plus the warp reductions the kernels share.  Every wait on an
// mbarrier is bounded: after kWaitLimitCycles the waiting warp records
// TQ_DEVERR_WAIT_TIMEOUT in the library's device error word and gives up,
// so a bad launch surfaces as an error status instead of a hung GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tq {

constexpr unsigned kFullMask = 0xffffffffu;

// ~1 s at the B200's 1.9 GHz SM clock.
constexpr long long kWaitLimitCycles = 2000000000LL;

// Bits of the device error word (read back by tq_device_status()).
enum DeviceError : int {
  TQ_DEVERR_WAIT_TIMEOUT = 1,  // an mbarrier wait ran out of time
  TQ_DEVERR_BAD_BLOCK = 2,     // a block id outside [0, num_blocks) reached a kernel
  TQ_DEVERR_BAD_SLOT = 4,      // a slot index outside the pool reached a kernel
  TQ_DEVERR_BAD_TOKEN = 8,     // a token id outside the vocabulary reached a kernel
  TQ_DEVERR_BAD_PLAN = 16,     // a work item's merge slot or split-K index lies outside its buffer
};

// The library is one translation unit (capi.cu includes every kernel
// header), so this definition is the only one.
__device__ int g_device_error = 0;

__device__ __forceinline__ void raise_device_error(int bits) { atomicOr(&g_device_error, bits); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Plain arrival (release at CTA scope): for barriers a thread, not TMA, completes.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for phase `parity` of `bar` to complete.  Returns false (and
// flags the error word) if it did not complete within kWaitLimitCycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) {
      raise_device_error(TQ_DEVERR_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ---- TMA bulk copy (untiled), global -> this CTA's shared memory -----------
// dst and src 16-byte aligned, bytes a multiple of 16.  Completion is reported
// to `bar` as transaction bytes.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Programmatic dependent launch.  launch_dependents: the next kernel in the
// stream, if launched with programmatic stream serialization, may start its
// CTAs (as resources free up) before this grid finishes.  wait: block until
// the preceding grid has completed and its memory is visible (returns at once
// when this kernel was not launched as a programmatic dependent).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- warp reductions --------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

}  // namespace tq
