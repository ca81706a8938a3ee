// The exported C ABI (include/cc1d.h): argument validation, scheduling and
// launches.  No entry point allocates, synchronises or keeps per-call state;
// the only process-wide state is a cache of device facts (SM count) and of
// kernel occupancies, both read-only after the first call.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "cc1d.h"
#include "cc1d_internal.h"

namespace cc1d {

namespace {

thread_local char g_err[512] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

thread_local char g_detail[160] = {0};

int cuda_fail(cudaError_t e, const char* what) {
  int dev = -1;
  (void)cudaGetDevice(&dev);
  (void)cudaGetLastError();  // the error is reported here, not by the next call
  fail(CC1D_ERR_CUDA, "%s: %s (%s) on device %d%s%s", what, cudaGetErrorString(e), cudaGetErrorName(e), dev,
       g_detail[0] ? ": " : "", g_detail);
  g_detail[0] = 0;
  return CC1D_ERR_CUDA;
}

// Device the calling thread was last bound to by bind_device.
thread_local int t_bound_device = -1;

// Makes the device that holds `ptr` current on the calling thread, with its
// primary context bound (the driver-level tensor-map encoder needs one).
// The caller's framework keeps its own runtime state and may never have
// bound a context on this thread (e.g. an autograd worker thread of device
// 0), so the device is taken from the data, not inherited.  Host or
// unregistered pointers leave the current device alone.
int bind_device(const void* ptr, const char* what) {
  if (ptr == nullptr) return CC1D_OK;
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, ptr);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return CC1D_OK;
  }
  if (at.type != cudaMemoryTypeDevice || at.device < 0) return CC1D_OK;
  int cur = -1;
  e = cudaGetDevice(&cur);
  if (e == cudaSuccess && (cur != at.device || t_bound_device != at.device)) {
    e = cudaSetDevice(at.device);  // initialises and binds the primary context
    if (e == cudaSuccess) t_bound_device = at.device;
  }
  return e == cudaSuccess ? CC1D_OK : cuda_fail(e, what);
}

int ok() {
  g_err[0] = 0;
  return CC1D_OK;
}

bool dtype_ok(int dt) { return dt == CC1D_F16 || dt == CC1D_BF16 || dt == CC1D_F32; }

// Width limits of causal_conv1d_fn (src/causal_conv1d_mojo/_fn.py:405-414).
int check_conv_width(int dtype, int width) {
  const int max_w = dtype == CC1D_F32 ? 5 : 9;
  if (width < 2 || width > max_w)
    return fail(CC1D_ERR_UNSUPPORTED, "width must be in 2..%d for this dtype (got %d)", max_w, width);
  return CC1D_OK;
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];
std::atomic<int> g_threads_per_sm[kMaxDevices];

}  // namespace

int report_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int report_cuda_error(cudaError_t e, const char* what) { return cuda_fail(e, what); }

void set_error_detail(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
  va_end(ap);
}

cudaError_t device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int sms = g_sms[dev].load(std::memory_order_relaxed);
  int tps = g_threads_per_sm[dev].load(std::memory_order_relaxed);
  if (sms <= 0) {
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&tps, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    if (e != cudaSuccess) return e;
    g_threads_per_sm[dev].store(tps, std::memory_order_relaxed);
    g_sms[dev].store(sms, std::memory_order_relaxed);
  }
  out->sms = sms;
  out->max_threads_per_sm = tps;
  return cudaSuccess;
}

namespace {

int fwd_args(const cc1d_fwd_params* p, FwdArgs* a) {
  if (p == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_fwd: params is NULL");
  if (!dtype_ok(p->dtype)) return fail(CC1D_ERR_UNSUPPORTED, "cc1d_fwd: unsupported dtype code %d", p->dtype);
  int rc = check_conv_width(p->dtype, p->width);
  if (rc) return rc;
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_fwd: negative shape (%lld, %lld, %lld)", (long long)p->batch,
                (long long)p->dim, (long long)p->seqlen);
  if (p->seq_idx && p->initial_states)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_fwd: seq_idx and initial_states are mutually exclusive");
  if (p->seq_idx && p->final_states)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_fwd: seq_idx and final_states are mutually exclusive");
  const bool work = p->batch * p->dim * p->seqlen > 0;
  if (work && (!p->x || !p->weight || !p->out))
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_fwd: x, weight and out are required");
  std::memset(a, 0, sizeof(*a));
  *a = FwdArgs{p->x, p->x_batch_stride, p->x_dim_stride, p->x_seq_stride,
               p->weight, p->weight_dim_stride, p->weight_width_stride,
               p->bias, p->bias_stride,
               p->seq_idx, p->seq_idx_batch_stride, p->seq_idx_seq_stride,
               p->initial_states, p->init_batch_stride, p->init_dim_stride, p->init_seq_stride,
               p->out, p->out_batch_stride, p->out_dim_stride, p->out_seq_stride,
               p->final_states, p->final_batch_stride, p->final_dim_stride, p->final_seq_stride,
               p->batch, p->dim, p->seqlen, p->silu ? 1 : 0,
               0, 0, 0, 0, 0};
  return CC1D_OK;
}

int bwd_args(const cc1d_bwd_params* p, BwdArgs* a) {
  if (p == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: params is NULL");
  if (!dtype_ok(p->dtype)) return fail(CC1D_ERR_UNSUPPORTED, "cc1d_bwd: unsupported dtype code %d", p->dtype);
  int rc = check_conv_width(p->dtype, p->width);
  if (rc) return rc;
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: negative shape");
  if (p->seq_idx && p->initial_states)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: seq_idx and initial_states are mutually exclusive");
  if (p->seq_idx && p->dfinal_states)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: seq_idx and dfinal_states are mutually exclusive");
  if (p->initial_states && !p->dinitial_states && p->batch * p->dim > 0)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: dinitial_states is required with initial_states");
  if (p->dim > 0 && !p->dwdb_acc) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: dwdb_acc is required");
  const bool work = p->batch * p->dim * p->seqlen > 0;
  if (work && (!p->x || !p->weight || !p->dout || !p->dx))
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd: x, weight, dout and dx are required");
  *a = BwdArgs{p->x, p->x_batch_stride, p->x_dim_stride, p->x_seq_stride,
               p->weight, p->weight_dim_stride, p->weight_width_stride,
               p->bias, p->bias_stride,
               p->dout, p->dout_batch_stride, p->dout_dim_stride, p->dout_seq_stride,
               p->seq_idx, p->seq_idx_batch_stride, p->seq_idx_seq_stride,
               p->initial_states, p->init_batch_stride, p->init_dim_stride, p->init_seq_stride,
               p->dfinal_states, p->dfinal_batch_stride, p->dfinal_dim_stride, p->dfinal_seq_stride,
               p->dx, p->dx_batch_stride, p->dx_dim_stride, p->dx_seq_stride,
               p->initial_states ? p->dinitial_states : nullptr, p->dinit_batch_stride, p->dinit_dim_stride,
               p->dinit_seq_stride,
               static_cast<float*>(p->workspace),
               p->batch, p->dim, p->seqlen, p->silu ? 1 : 0,
               0, 0, 0, 0, 0};
  return CC1D_OK;
}

// Backward kernel family: 2 = TMA along seqlen, 1 = TMA along dim, 0 =
// register streaming.  The workspace size depends on it, so the size query
// and the launch must agree (both go through here).
int bwd_family(int dtype, const BwdArgs& a) {
  return bwd_seq_tma_eligible(dtype, a) ? 2 : (bwd_tma_eligible(dtype, a) ? 1 : 0);
}

cudaError_t plan_bwd_any(int dtype, int width, const BwdArgs& a, Plan* plan) {
  const int fam = bwd_family(dtype, a);
  return fam == 2 ? plan_bwd_seq_tma(dtype, width, a, plan)
                  : fam == 1 ? plan_bwd_tma(dtype, width, a, plan) : plan_bwd(dtype, width, a, plan);
}

// Workspace of a backward plan: the dweight/dbias partials, then (256-byte
// aligned) the plan's auxiliary bytes.
size_t workspace_bytes(const Plan& plan, int64_t dim, int width) {
  const size_t partials = (size_t)plan.n_partials * (size_t)dim * (size_t)(width + 1) * sizeof(float);
  if (plan.aux_bytes == 0) return partials;
  return (partials + 255) / 256 * 256 + (size_t)plan.aux_bytes;
}

}  // namespace
}  // namespace cc1d

using namespace cc1d;

extern "C" {

int cc1d_fwd(const cc1d_fwd_params* p, void* stream) {
  FwdArgs a;
  int rc = fwd_args(p, &a);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->batch * p->dim == 0) return ok();
  if ((rc = bind_device(p->out, "cc1d_fwd")) != CC1D_OK) return rc;
  if (p->seqlen == 0) {
    cudaError_t e = launch_fwd_empty_seq(p->dtype, p->width, a, s);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cc1d_fwd (empty sequence)");
  }
  Plan plan;
  std::memset(&plan, 0, sizeof(plan));
  // Kernel family: TMA pipeline along seqlen, TMA pipeline along dim
  // (channel-last), else register streaming (any strides).
  const int fam = fwd_seq_tma_eligible(p->dtype, a) ? 2 : (fwd_tma_eligible(p->dtype, a) ? 1 : 0);
  cudaError_t e = fam == 2   ? plan_fwd_seq_tma(p->dtype, p->width, a, &plan)
                  : fam == 1 ? plan_fwd_tma(p->dtype, p->width, a, &plan)
                             : plan_fwd(p->dtype, p->width, a, &plan);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_fwd plan");
  e = fam == 2   ? launch_fwd_seq_tma(p->dtype, p->width, a, plan, s)
      : fam == 1 ? launch_fwd_tma(p->dtype, p->width, a, plan, s)
                 : launch_fwd(p->dtype, p->width, a, plan, s);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_fwd launch");
  return ok();
}

int cc1d_bwd_workspace_size(const cc1d_bwd_params* p, size_t* bytes) {
  if (bytes == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_workspace_size: bytes is NULL");
  *bytes = 0;
  BwdArgs a;
  int rc = bwd_args(p, &a);
  if (rc) return rc;
  if (p->batch * p->dim * p->seqlen == 0) return ok();
  if ((rc = bind_device(p->dwdb_acc, "cc1d_bwd_workspace_size")) != CC1D_OK) return rc;
  Plan plan;
  std::memset(&plan, 0, sizeof(plan));
  cudaError_t e = plan_bwd_any(p->dtype, p->width, a, &plan);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd plan");
  *bytes = workspace_bytes(plan, p->dim, p->width);
  return ok();
}

}  // extern "C"

namespace {

// cc1d_bwd, optionally with the dweight/dbias reduction fused with a
// cross-GPU all-reduce (peer != nullptr).
int bwd_impl(const cc1d_bwd_params* p, const cc1d_peer_reduce* peer, void* stream) {
  BwdArgs a;
  int rc = bwd_args(p, &a);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned mode = peer != nullptr ? peer->flags : CC1D_PEER_FUSED;
  if (peer != nullptr) {
    if (peer->world < 1 || peer->rank < 0 || peer->rank >= peer->world || peer->world > 32)
      return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_peer_reduce: rank %d / world %d invalid (world <= 32)",
                  peer->rank, peer->world);
    if (p->dim > 0 && (!peer->exchange || !peer->epochs))
      return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_peer_reduce: exchange and epochs are required");
    if (mode != CC1D_PEER_FUSED && mode != CC1D_PEER_PUSH && mode != CC1D_PEER_FINISH)
      return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_peer_reduce: unknown flags %u", mode);
  }
  if (p->dim == 0) return ok();
  if ((rc = bind_device(p->dwdb_acc, "cc1d_bwd")) != CC1D_OK) return rc;
  Plan plan;
  std::memset(&plan, 0, sizeof(plan));
  cudaError_t e = cudaSuccess;
  if (mode == CC1D_PEER_FINISH) {
    // Second half of a split exchange: only the wait and the outputs.
    FinalizeArgs f{nullptr, 0, p->dim, p->dwdb_acc, p->dweight_out, p->dweight_dim_stride, p->dweight_width_stride,
                   p->dbias_out, p->dbias_stride, p->bias != nullptr ? 1 : 0};
    PeerFinalizeArgs pf{f, peer->rank, peer->world, peer->exchange, peer->epochs, peer_blocks(p->dim, p->width),
                        peer->max_polls != 0 ? peer->max_polls : 4194304u, peer->status};
    e = launch_finalize_peer(p->dtype, p->width, pf, 2, s);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cc1d_bwd_peer_reduce finish launch");
  }
  if (p->batch * p->seqlen > 0) {
    const int fam = bwd_family(p->dtype, a);
    e = plan_bwd_any(p->dtype, p->width, a, &plan);
    if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd plan");
    const size_t need = workspace_bytes(plan, p->dim, p->width);
    if (need > 0 && (p->workspace == nullptr || p->workspace_bytes < need))
      return fail(CC1D_ERR_WORKSPACE, "cc1d_bwd: workspace of %zu bytes needed, %zu given", need,
                  p->workspace == nullptr ? (size_t)0 : p->workspace_bytes);
    e = fam == 2   ? launch_bwd_seq_tma(p->dtype, p->width, a, plan, s)
        : fam == 1 ? launch_bwd_tma(p->dtype, p->width, a, plan, s)
                   : launch_bwd(p->dtype, p->width, a, plan, s);
    if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd launch");
  } else if (p->batch > 0 && p->seqlen == 0) {
    e = launch_bwd_empty_seq(p->dtype, p->width, a, s);
    if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd (empty sequence)");
  }
  FinalizeArgs f{static_cast<const float*>(p->workspace), plan.n_partials, p->dim, p->dwdb_acc,
                 p->dweight_out, p->dweight_dim_stride, p->dweight_width_stride,
                 p->dbias_out, p->dbias_stride, p->bias != nullptr ? 1 : 0};
  if (peer == nullptr) {
    e = launch_finalize(p->dtype, p->width, f, s);
    if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd finalize launch");
  } else {
    PeerFinalizeArgs pf{f, peer->rank, peer->world, peer->exchange, peer->epochs, peer_blocks(p->dim, p->width),
                        peer->max_polls != 0 ? peer->max_polls : 4194304u, peer->status};
    e = launch_finalize_peer(p->dtype, p->width, pf, mode == CC1D_PEER_PUSH ? 1 : 0, s);
    if (e != cudaSuccess) return cuda_fail(e, "cc1d_bwd_peer_reduce finalize launch");
  }
  return ok();
}

}  // namespace

extern "C" {

int cc1d_bwd(const cc1d_bwd_params* p, void* stream) { return bwd_impl(p, nullptr, stream); }

int cc1d_bwd_peer_reduce(const cc1d_bwd_params* p, const cc1d_peer_reduce* peer, void* stream) {
  if (peer == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_bwd_peer_reduce: peer is NULL");
  return bwd_impl(p, peer, stream);
}

int64_t cc1d_peer_blocks(int64_t dim, int32_t width) { return dim <= 0 ? 0 : peer_blocks(dim, width); }

int64_t cc1d_peer_exchange_bytes(int64_t dim, int32_t width, int32_t world) {
  return dim <= 0 || world <= 0 ? 0 : peer_exchange_bytes(dim, width, world);
}

int cc1d_update(const cc1d_update_params* p, void* stream) {
  if (p == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_update: params is NULL");
  if (!dtype_ok(p->dtype)) return fail(CC1D_ERR_UNSUPPORTED, "cc1d_update: unsupported dtype code %d", p->dtype);
  // Width limits of causal_conv1d_update (src/causal_conv1d_mojo/_update.py:109-115).
  if (p->width < 2 || p->width > 9)
    return fail(CC1D_ERR_UNSUPPORTED, "width must be in 2..9 (got %d)", p->width);
  if (p->batch < 0 || p->dim < 0 || p->seqlen < 0 || p->state_len < 0)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_update: negative shape");
  if (p->state_len < p->width - 1)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "conv_state.shape[-1]=%lld must be >= width-1=%d",
                (long long)p->state_len, p->width - 1);
  if (p->batch * p->dim == 0) return ok();
  if (!p->x || !p->weight || !p->conv_state || !p->out)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_update: x, weight, conv_state and out are required");
  if (p->conv_state_indices == nullptr && p->state_rows < p->batch)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_update: conv_state has %lld rows for batch %lld",
                (long long)p->state_rows, (long long)p->batch);
  int rc = bind_device(p->out, "cc1d_update");
  if (rc != CC1D_OK) return rc;
  UpdateArgs a{p->x, p->x_batch_stride, p->x_dim_stride, p->x_seq_stride,
               p->weight, p->weight_dim_stride, p->weight_width_stride,
               p->bias, p->bias_stride,
               p->conv_state, p->state_batch_stride, p->state_dim_stride, p->state_seq_stride,
               p->conv_state_indices, p->cache_seqlens,
               p->out, p->out_batch_stride, p->out_dim_stride, p->out_seq_stride,
               p->batch, p->dim, p->seqlen, p->state_len, p->state_rows, p->silu ? 1 : 0};
  cudaError_t e = launch_update(p->dtype, p->width, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_update launch");
  return ok();
}

int cc1d_varlen_states(const cc1d_varlen_states_params* p, void* stream) {
  if (p == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_varlen_states: params is NULL");
  if (!dtype_ok(p->dtype))
    return fail(CC1D_ERR_UNSUPPORTED, "cc1d_varlen_states: unsupported dtype code %d", p->dtype);
  if (p->batch < 0 || p->dim < 0 || p->state_len < 0 || p->total_tokens < 0)
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_varlen_states: negative shape");
  if (p->batch * p->dim * p->state_len == 0) return ok();
  if (!p->cu_seqlens || !p->states || (!p->x && p->total_tokens > 0))
    return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_varlen_states: x, cu_seqlens and states are required");
  int rc = bind_device(p->states, "cc1d_varlen_states");
  if (rc != CC1D_OK) return rc;
  VarlenArgs a{p->x, p->x_token_stride, p->x_dim_stride, p->cu_seqlens,
               p->states, p->states_batch_stride, p->states_dim_stride, p->states_seq_stride,
               p->batch, p->dim, p->state_len, p->total_tokens};
  cudaError_t e = launch_varlen_states(p->dtype, a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_varlen_states launch");
  return ok();
}

int cc1d_device_status(unsigned* wait_timeouts) {
  if (wait_timeouts == nullptr) return fail(CC1D_ERR_INVALID_ARGUMENT, "cc1d_device_status: NULL output");
  cudaError_t e = read_wait_timeouts(wait_timeouts);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_device_status");
  e = read_peer_timeouts(wait_timeouts);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_device_status");
  e = read_fused_aborts(wait_timeouts);
  if (e != cudaSuccess) return cuda_fail(e, "cc1d_device_status");
  return ok();
}

const char* cc1d_last_error(void) { return g_err; }

const char* cc1d_version(void) { return "1.6.1"; }

int cc1d_abi_version(void) { return CC1D_ABI_VERSION; }

}  // extern "C"
