// cc1d_bwd_noalloc: the fused backward for callers that cannot allocate
// device memory for the per-call scratch that cc1d_bwd takes as `workspace`.
//
// Who needs it: code that runs where cudaMalloc is unavailable or harmful --
// a serving engine that reserved nearly all of HBM up front (so a new
// allocation fails), a caller bound through a foreign-function interface
// with no access to the host framework's allocator, or a latency-critical
// loop where cudaMalloc's implicit device synchronisation is not allowed.
//
// The scratch lives in a file-scope static device array of
// CC1D_NOALLOC_SCRATCH_BYTES (16 MiB).  Every GPU that loads this library
// holds that array until the process exits.  The device address of the
// array is obtained once per device, on the first call made with that
// device current (cudaGetSymbolAddress), and cached; make that first call
// before any stream capture.  Every call shares the array and it keeps the
// previous call's contents: the backward overwrites every partial-sum slot
// it reads, so nothing needs clearing, but calls whose executions overlap on
// the GPU (different streams, or concurrent host threads) race on it.
#include <atomic>

#include "cc1d.h"
#include "cc1d_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_bwd_scratch[CC1D_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_addr[kMaxDevices];

// Device address of g_bwd_scratch on the current device (cached per device).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cc1d::report_cuda_error(e, "cc1d_bwd_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return cc1d::report_error(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_noalloc: device %d out of range", dev);
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess) return cc1d::report_cuda_error(e, "cc1d_bwd_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return CC1D_OK;
}

}  // namespace

extern "C" int cc1d_bwd_noalloc(const cc1d_bwd_params* params, void* stream) {
  if (params == nullptr) return cc1d::report_error(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_noalloc: params is NULL");
  cc1d_bwd_params p = *params;
  p.workspace = nullptr;
  p.workspace_bytes = 0;
  size_t need = 0;
  int rc = cc1d_bwd_workspace_size(&p, &need);
  if (rc != CC1D_OK) return rc;
  if (need > (size_t)CC1D_NOALLOC_SCRATCH_BYTES)
    return cc1d::report_error(CC1D_ERR_WORKSPACE,
                              "cc1d_bwd_noalloc: this call needs %zu bytes of scratch but the built-in scratch "
                              "holds %zu bytes; use cc1d_bwd with a caller-provided workspace",
                              need, (size_t)CC1D_NOALLOC_SCRATCH_BYTES);
  if (need > 0) {
    // cc1d_bwd_workspace_size made the device holding the data current on
    // this thread (it does so whenever the call has work, i.e. need > 0),
    // so the symbol address is that device's copy of the array.  Calls with
    // nothing to reduce take no scratch and never look it up: they cannot
    // touch, or cache the address on, whatever device happens to be current.
    void* scratch = nullptr;
    rc = scratch_address(&scratch);
    if (rc != CC1D_OK) return rc;
    p.workspace = scratch;
    p.workspace_bytes = CC1D_NOALLOC_SCRATCH_BYTES;
  }
  return cc1d_bwd(&p, stream);
}
