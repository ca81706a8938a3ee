// Internal (non-exported) interface between the C ABI layer (cc1d_abi.cu)
// and the kernel translation units.  Strides are in elements, 64-bit.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cc1d {

typedef int64_t i64;

// How a (batch, dim, seqlen) tensor is walked.
//   kSeq:  the seqlen axis is the vector axis (x.stride(2) == 1); one warp
//          walks a segment of one (b, c) row, each lane owning 16 bytes.
//   kChan: the dim axis is the vector axis (x.stride(1) == 1, channel-last);
//          each lane owns a few adjacent channels and walks time.
enum Layout { kSeq = 0, kChan = 1 };

struct Plan {
  Layout layout;
  bool vec;        // vector loads/stores allowed (unit stride + alignment)
  int threads;     // block size
  i64 grid;        // number of blocks
  // kSeq: items = rows * nseg, each a segment of seg_len timesteps.
  i64 nseg, seg_len, n_items;
  // kChan: block = (channel group, split); split covers rows_per_split
  // flattened (b, t) rows of one channel group.
  i64 groups, splits, rows_per_split;
  // Backward: number of partial (dweight|dbias) sets per channel.
  i64 n_partials;
  // Backward: bytes of workspace after the partials (256-byte aligned) for
  // per-position data a kernel family derives from its inputs first (the
  // seqlen kernels' sequence masks with seq_idx); 0 when none.
  i64 aux_bytes;
};

struct FwdArgs {
  const void* x; i64 xs_b, xs_c, xs_l;
  const void* w; i64 ws_c, ws_k;
  const void* bias; i64 bs;
  const int* seq; i64 ss_b, ss_l;
  const void* init; i64 is_b, is_c, is_l;
  void* out; i64 os_b, os_c, os_l;
  void* fin; i64 fs_b, fs_c, fs_l;
  i64 B, D, L;
  int silu;
  // schedule (copied from Plan)
  i64 nseg, seg_len, n_items;
  i64 splits, rows_per_split;
};

struct BwdArgs {
  const void* x; i64 xs_b, xs_c, xs_l;
  const void* w; i64 ws_c, ws_k;
  const void* bias; i64 bs;
  const void* dout; i64 gs_b, gs_c, gs_l;
  const int* seq; i64 ss_b, ss_l;
  const void* init; i64 is_b, is_c, is_l;
  const void* dfin; i64 fs_b, fs_c, fs_l;
  void* dx; i64 dxs_b, dxs_c, dxs_l;
  void* dinit; i64 dis_b, dis_c, dis_l;
  float* partials;  // [n_partials][D][W+1]
  i64 B, D, L;
  int silu;
  i64 nseg, seg_len, n_items;
  i64 splits, rows_per_split;
};

struct FinalizeArgs {
  const float* partials; i64 n_partials;
  i64 D;
  float* dwdb;                      // [D*W | D]
  void* dw_out; i64 dws_c, dws_k;   // optional, dtype
  void* db_out; i64 dbs;            // optional, dtype
  int has_bias;
};

// Cross-GPU reduction of the dweight/dbias partials (cc1d_peer.cu).
struct PeerFinalizeArgs {
  FinalizeArgs f;
  int rank, world;
  unsigned long long* const* bufs;  // device array [world] of exchange buffers
  uint32_t* epochs;                 // this rank's per-block call counters (nblocks)
  i64 nblocks;
  unsigned max_polls;               // bounded wait per peer word
  uint32_t* status;                 // optional: +1 per warp whose wait gave up
};

struct UpdateArgs {
  const void* x; i64 xs_b, xs_c, xs_l;
  const void* w; i64 ws_c, ws_k;
  const void* bias; i64 bs;
  void* state; i64 ss_b, ss_c, ss_l;
  const int* idx;
  const int* cache_seqlens;
  void* out; i64 os_b, os_c, os_l;
  i64 B, D, L, S;
  i64 state_rows;  // rows of conv_state; indices outside [0, rows) act as padding
  int silu;
};

struct VarlenArgs {
  const void* x; i64 xs_t, xs_c;
  const int* cu;
  void* st; i64 ss_b, ss_c, ss_l;
  i64 B, D, S;
  i64 total_tokens;  // rows of x; reads outside [0, total_tokens) give 0
};

// Device facts used for scheduling (cached per device).
struct DeviceInfo {
  int sms;
  int max_threads_per_sm;
};
cudaError_t device_info(DeviceInfo* out);

// Kernel-family launchers; each returns the launch error (if any).
// plan_* fill the schedule (grid, splits, ...) for the given shapes.
cudaError_t plan_fwd(int dtype, int width, const FwdArgs& a, Plan* plan);
cudaError_t launch_fwd(int dtype, int width, FwdArgs a, const Plan& plan, cudaStream_t stream);

cudaError_t plan_bwd(int dtype, int width, const BwdArgs& a, Plan* plan);
cudaError_t launch_bwd(int dtype, int width, BwdArgs a, const Plan& plan, cudaStream_t stream);
cudaError_t launch_finalize(int dtype, int width, const FinalizeArgs& a, cudaStream_t stream);
// Length-0 sequences: dinitial_states = dfinal_states (or 0).
cudaError_t launch_bwd_empty_seq(int dtype, int width, const BwdArgs& a, cudaStream_t stream);
// Length-0 sequences: final_states = initial_states (or 0).
cudaError_t launch_fwd_empty_seq(int dtype, int width, const FwdArgs& a, cudaStream_t stream);

// TMA-pipelined channel-last kernels (cc1d_chan_tma.cu); used when the
// strides and alignment allow tensor-map tile loads.
bool fwd_tma_eligible(int dtype, const FwdArgs& a);
cudaError_t plan_fwd_tma(int dtype, int width, const FwdArgs& a, Plan* plan);
cudaError_t launch_fwd_tma(int dtype, int width, const FwdArgs& a, const Plan& plan, cudaStream_t stream);
bool bwd_tma_eligible(int dtype, const BwdArgs& a);
cudaError_t plan_bwd_tma(int dtype, int width, const BwdArgs& a, Plan* plan);
cudaError_t launch_bwd_tma(int dtype, int width, const BwdArgs& a, const Plan& plan, cudaStream_t stream);

// TMA-pipelined seqlen-contiguous kernels (cc1d_seq_tma.cu).
bool fwd_seq_tma_eligible(int dtype, const FwdArgs& a);
cudaError_t plan_fwd_seq_tma(int dtype, int width, const FwdArgs& a, Plan* plan);
cudaError_t launch_fwd_seq_tma(int dtype, int width, const FwdArgs& a, const Plan& plan, cudaStream_t stream);
bool bwd_seq_tma_eligible(int dtype, const BwdArgs& a);
cudaError_t plan_bwd_seq_tma(int dtype, int width, const BwdArgs& a, Plan* plan);
cudaError_t launch_bwd_seq_tma(int dtype, int width, const BwdArgs& a, const Plan& plan, cudaStream_t stream);
cudaError_t read_seq_wait_timeouts(unsigned* count);

i64 peer_blocks(i64 dim, int width);
i64 peer_exchange_bytes(i64 dim, int width, int world);
// mode: 0 the fused exchange, 1 push only, 2 finish only (cc1d_peer.cu).
cudaError_t launch_finalize_peer(int dtype, int width, const PeerFinalizeArgs& p, int mode, cudaStream_t stream);
cudaError_t read_peer_timeouts(unsigned* count);
// Blocks of the fused in_proj + conv kernel that gave up on a bounded wait.
cudaError_t read_fused_aborts(unsigned* count);

// Records a message for cc1d_last_error() and returns `code` (for entry
// points defined outside cc1d_abi.cu).
int report_error(int code, const char* fmt, ...);
int report_cuda_error(cudaError_t e, const char* what);
// Extra text for the next CUDA error message of this thread (e.g. why a
// tensor map could not be encoded).
void set_error_detail(const char* fmt, ...);

// Reads and clears the device-side count of bounded waits that gave up.
cudaError_t read_wait_timeouts(unsigned* count);

cudaError_t launch_update(int dtype, int width, const UpdateArgs& a, cudaStream_t stream);
cudaError_t launch_varlen_states(int dtype, const VarlenArgs& a, cudaStream_t stream);

}  // namespace cc1d
