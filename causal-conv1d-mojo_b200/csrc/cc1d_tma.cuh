// TMA (cp.async.bulk.tensor) and mbarrier primitives for the pipelined
// kernels, as inline PTX for sm_100a.
//
// Only plain (non-multicast) tile loads from this GPU's own memory are used.
// Every wait on an mbarrier is bounded: after kSpinLimit failed polls the
// wait gives up, the kernel counts the event in g_cc1d_wait_timeouts (read
// by cc1d_device_status) and the caller returns instead of hanging.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "cc1d_common.cuh"

namespace cc1d {

// Polls of mbarrier.try_wait before a wait gives up.  try_wait itself
// suspends for a hardware-chosen interval, so this is well over a second.
constexpr unsigned kSpinLimit = 1u << 22;

// Number of bounded waits that gave up since the last read.  One counter per
// translation unit that includes this header (no relocatable device code);
// each such unit reads and clears its own with tu_read_wait_timeouts().
static __device__ unsigned int g_cc1d_wait_timeouts = 0;

static inline cudaError_t tu_read_wait_timeouts(unsigned* count) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_cc1d_wait_timeouts, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  *count += v;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_cc1d_wait_timeouts, &zero, sizeof(unsigned));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicAdd(&g_cc1d_wait_timeouts, 1u);
  return false;
}

// Producer epilogue of a `stages`-deep ring into which `issued` stage loads
// were issued (stage k % stages, phase k / stages): waits, bounded, for the
// last min(issued, stages) of them to land.  In the normal flow they have
// landed or are about to (the consumers wait for the same phases).  After a
// wait gave up -- the consumers may have returned -- it keeps this block
// resident until its bulk copies stop writing its shared memory, so no
// block exits with async copies still in flight.  Stops at the first wait
// that gives up (counted like any other).
__device__ __forceinline__ void mbar_drain(uint64_t* full, unsigned issued, unsigned stages) {
  const unsigned n = issued < stages ? issued : stages;
  for (unsigned i = 1; i <= n; ++i) {
    const unsigned k = issued - i;
    if (!mbar_wait(&full[k % stages], (k / stages) & 1)) return;
  }
}

// 3-D tiled TMA load into shared memory, completion signalled on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace cc1d
