// Compile-time dispatch over (dtype, width) and occupancy-based grid sizing.
#pragma once

#include <atomic>
#include <utility>

#include "cc1d_common.cuh"
#include "cc1d_internal.h"

namespace cc1d {

// Calls f.template operator()<T, W>() for the runtime (dtype, width).
// Widths whose halo (W-1) does not fit one 16-byte lane vector are not
// instantiated (fp32 stops at W=5; fp16/bf16 at W=9).
template <typename T, typename F>
cudaError_t dispatch_width(int width, F&& f) {
  constexpr int V = 16 / (int)sizeof(T);
  switch (width) {
    case 2: return f.template operator()<T, 2>();
    case 3: return f.template operator()<T, 3>();
    case 4: return f.template operator()<T, 4>();
    case 5: return f.template operator()<T, 5>();
    case 6: if constexpr (V >= 5) return f.template operator()<T, 6>(); break;
    case 7: if constexpr (V >= 6) return f.template operator()<T, 7>(); break;
    case 8: if constexpr (V >= 7) return f.template operator()<T, 8>(); break;
    case 9: if constexpr (V >= 8) return f.template operator()<T, 9>(); break;
    default: break;
  }
  return cudaErrorInvalidValue;
}

template <typename F>
cudaError_t dispatch(int dtype, int width, F&& f) {
  switch (dtype) {
    case 0: return dispatch_width<__half>(width, f);
    case 1: return dispatch_width<__nv_bfloat16>(width, f);
    case 2: return dispatch_width<float>(width, f);
    default: return cudaErrorInvalidValue;
  }
}

// Launch with programmatic stream serialization (PDL): the kernel may be
// scheduled while the previous kernel in the stream drains, and must call
// griddep_wait() before touching global memory.  Captured into CUDA graphs
// as a programmatic edge.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Resident blocks per SM for `kernel` at `threads` threads and `smem` bytes
// of dynamic shared memory; cached per call site (per template instance).
template <typename K>
cudaError_t blocks_per_sm(K kernel, int threads, size_t smem, std::atomic<int>& cache, int* out) {
  int v = cache.load(std::memory_order_relaxed);
  if (v <= 0) {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, kernel, threads, smem);
    if (e != cudaSuccess) return e;
    if (v < 1) v = 1;
    cache.store(v, std::memory_order_relaxed);
  }
  *out = v;
  return cudaSuccess;
}

}  // namespace cc1d
