/*
 * cc1d.h -- C ABI of the B200 (sm_100a) causal depthwise conv1d library
 * (libcc1d_sm100.so).
 *
 * The reference (causal-conv1d-mojo) crosses its native boundary with a
 * positional Python tuple of integers per op: data pointers (0 for an absent
 * tensor), B/D/L, per-tensor strides in elements, flags, a dtype code and the
 * caller's CUDA stream.  This header replaces those tuples with one plain C
 * struct per op.  Every pointer is a device address, every stride is counted
 * in ELEMENTS (not bytes) and is 64-bit, so tensors with more than 2^31
 * elements are addressed correctly.
 *
 * Conventions shared by every entry point:
 *   - All work is enqueued on `stream` (a cudaStream_t, may be 0 for the
 *     legacy default stream) of the CURRENT CUDA device.  No entry point
 *     synchronises, allocates device memory or keeps state between calls.
 *   - Return value: CC1D_OK (0) or a CC1D_ERR_* code.  The matching message
 *     is available from cc1d_last_error() on the calling thread.
 *   - A tensor with zero elements launches nothing and returns CC1D_OK.
 *   - dtype codes equal the reference's (_dtype.py:16-20): fp16=0, bf16=1,
 *     fp32=2.
 */
#ifndef CC1D_H_
#define CC1D_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CC1D_ABI_VERSION 2

#if defined(__GNUC__)
#define CC1D_API __attribute__((visibility("default")))
#else
#define CC1D_API
#endif

enum cc1d_dtype { CC1D_F16 = 0, CC1D_BF16 = 1, CC1D_F32 = 2 };

enum cc1d_status {
  CC1D_OK = 0,
  CC1D_ERR_INVALID_ARGUMENT = 1, /* bad shape / stride / pointer / flag */
  CC1D_ERR_UNSUPPORTED = 2,      /* width or dtype outside the supported set */
  CC1D_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
  CC1D_ERR_WORKSPACE = 4         /* workspace missing or too small */
};

/*
 * Forward pass of causal_conv1d_fn.
 *   out[b,c,t] = act(bias[c] + sum_{k<W} weight[c,k] * xc[b,c,t-(W-1)+k])
 * where xc is x preceded by initial_states (or by zeros), act is SiLU when
 * `silu` != 0, and with seq_idx a tap is used only when
 * seq_idx[b,src] == seq_idx[b,t]; seq_idx[b,t] < 0 forces out = 0.
 * final_states (optional) receives the last W-1 columns of
 * cat([initial_states or zeros, x], -1) bit-exactly.
 *
 * Replaces the 29-tuple built by `native_fwd`
 * (src/causal_conv1d_mojo/fwd/__init__.py:27-59) plus the torch copy in
 * `_write_final_states` (src/causal_conv1d_mojo/_fn.py:31-50).
 */
typedef struct cc1d_fwd_params {
  int32_t dtype;   /* enum cc1d_dtype; x, weight, bias, states and out share it */
  int32_t width;   /* W: 2..9 for fp16/bf16, 2..5 for fp32 */
  int64_t batch, dim, seqlen;
  int32_t silu;    /* 1: SiLU (= swish) activation, 0: none */
  int32_t _pad0;
  const void* x;            int64_t x_batch_stride, x_dim_stride, x_seq_stride;
  const void* weight;       int64_t weight_dim_stride, weight_width_stride;
  const void* bias;         int64_t bias_stride;          /* NULL: no bias */
  const int32_t* seq_idx;   int64_t seq_idx_batch_stride, seq_idx_seq_stride; /* NULL: none */
  const void* initial_states; int64_t init_batch_stride, init_dim_stride, init_seq_stride; /* NULL: zeros */
  void* out;                int64_t out_batch_stride, out_dim_stride, out_seq_stride;
  void* final_states;       int64_t final_batch_stride, final_dim_stride, final_seq_stride; /* NULL: not written */
} cc1d_fwd_params;

CC1D_API int cc1d_fwd(const cc1d_fwd_params* params, void* stream);

/*
 * Fused backward of causal_conv1d_fn: recomputes the pre-activation and
 * produces dx, dinitial_states (when initial_states is given), and the fp32
 * weight/bias gradient sums.  dfinal_states (optional) is folded into dx and
 * dinitial_states, so no separate tail-add is needed.
 *
 * dweight/dbias: the kernel writes per-block partial sums into `workspace`
 * (size from cc1d_bwd_workspace_size) and a second kernel reduces them in a
 * fixed order -- results are bitwise reproducible run to run.  With seq_idx
 * on seqlen-contiguous data the workspace also holds per-position sequence
 * masks that a first kernel derives from seq_idx.  The reduced
 * fp32 sums are OVERWRITTEN (not accumulated) into `dwdb_acc`, a contiguous
 * fp32 buffer of dim*(W+1) floats laid out as [dweight (dim, W) | dbias (dim)]
 * so that one all-reduce covers both when the batch is sharded across GPUs.
 * Optionally the same sums are also written rounded to `dtype` into
 * `dweight_out` / `dbias_out`.
 *
 * Replaces the 39-tuple built by `native_bwd_full`
 * (src/causal_conv1d_mojo/bwd_full/__init__.py:150-193) and the Python
 * post-processing in `_CausalConv1dFn.backward`
 * (src/causal_conv1d_mojo/_fn.py:274-332: dout.contiguous(), zeroed fp32
 * accumulators, the dfinal_states tail add and the dtype casts).
 */
typedef struct cc1d_bwd_params {
  int32_t dtype;
  int32_t width;
  int64_t batch, dim, seqlen;
  int32_t silu;
  int32_t _pad0;
  const void* x;            int64_t x_batch_stride, x_dim_stride, x_seq_stride;
  const void* weight;       int64_t weight_dim_stride, weight_width_stride;
  const void* bias;         int64_t bias_stride;          /* NULL: no bias (dbias not produced) */
  const void* dout;         int64_t dout_batch_stride, dout_dim_stride, dout_seq_stride;
  const int32_t* seq_idx;   int64_t seq_idx_batch_stride, seq_idx_seq_stride;
  const void* initial_states; int64_t init_batch_stride, init_dim_stride, init_seq_stride;
  const void* dfinal_states;  int64_t dfinal_batch_stride, dfinal_dim_stride, dfinal_seq_stride; /* NULL: none */
  void* dx;                 int64_t dx_batch_stride, dx_dim_stride, dx_seq_stride;
  void* dinitial_states;    int64_t dinit_batch_stride, dinit_dim_stride, dinit_seq_stride; /* required iff initial_states */
  float* dwdb_acc;          /* required: dim*(W+1) fp32, contiguous */
  void* dweight_out;        int64_t dweight_dim_stride, dweight_width_stride; /* NULL: skip */
  void* dbias_out;          int64_t dbias_stride;        /* NULL: skip */
  void* workspace;          size_t workspace_bytes;
} cc1d_bwd_params;

/* Bytes of scratch cc1d_bwd needs for `params` (only shapes, dtype, width and
 * strides are read).  Writes 0 to *bytes when the call would launch nothing. */
CC1D_API int cc1d_bwd_workspace_size(const cc1d_bwd_params* params, size_t* bytes);

CC1D_API int cc1d_bwd(const cc1d_bwd_params* params, void* stream);

/*
 * cc1d_bwd for a batch-sharded job on several GPUs: identical, except that
 * the final dweight/dbias reduction is fused with the all-reduce across the
 * `world` ranks, through NVLink peer memory, in one kernel.  On return (in
 * stream order) every rank's dwdb_acc / dweight_out / dbias_out hold the
 * sums over all ranks' batch shards -- bitwise identical on all ranks,
 * added in rank order.  Replaces the NCCL all-reduce of the fp32 buffer that
 * a batch-sharded use of the reference's causal_conv1d_fn would need (the
 * reference has no multi-GPU code).
 *
 * exchange[r]: rank r's exchange buffer, mapped into this process (e.g. by
 * CUDA IPC), cc1d_peer_exchange_bytes(dim, W, world) bytes, zero before the
 * first call; every rank stores into every other rank's buffer.  epochs:
 * this rank's cc1d_peer_blocks(dim, W) uint32 call counters, zero before
 * the first call, advanced on the device by every call (so the call may be
 * captured in a CUDA graph and replayed).  All ranks must issue the same
 * sequence of calls with the same dim and W, one rank per GPU.  Waits for
 * peers are bounded.  A wait that gives up (a peer that is late by more than
 * max_polls polls, or gone) writes NaN into the dwdb_acc / dweight_out /
 * dbias_out elements it could not reduce -- never stale values -- adds 1 to
 * *status (when given) and to the count cc1d_device_status reports.  The
 * call numbers still advance, so the ranks stay in step for the next call.
 *
 * Split exchange (flags): CC1D_PEER_PUSH runs the backward and the first half
 * of the reduction only -- the local sums are pushed to every rank and the
 * call returns without waiting; dwdb_acc / dweight_out / dbias_out are not
 * written.  A later call with CC1D_PEER_FINISH and the same params (nothing
 * but the reduction runs: no backward, no workspace) waits for the ranks'
 * sums and writes the outputs.  Issue FINISH on another stream to overlap the
 * wait for the slowest rank with other work, and order each FINISH before
 * the same rank's next PUSH (e.g. the PUSH stream waits on an event recorded
 * after FINISH).  Split calls count on their own epochs array: 4 zeroed
 * uint32 words shared by the PUSH and FINISH calls of one reducer, which
 * must not also make fused calls (flags 0) on the same exchange buffers.
 */
#define CC1D_PEER_FUSED 0u
#define CC1D_PEER_PUSH 1u
#define CC1D_PEER_FINISH 2u

typedef struct cc1d_peer_reduce {
  int32_t rank, world;                 /* world <= 32 */
  unsigned long long* const* exchange; /* device array [world] */
  uint32_t* epochs;                    /* this rank's counters */
  uint32_t max_polls;                  /* polls per wait before giving up; 0 = 4194304 (seconds) */
  uint32_t flags;                      /* CC1D_PEER_FUSED (0), CC1D_PEER_PUSH or CC1D_PEER_FINISH */
  uint32_t* status;                    /* device word, or NULL: +1 per wait that gave up (the caller
                                          zeroes it and reads it at a sync point of its choosing) */
} cc1d_peer_reduce;

CC1D_API int64_t cc1d_peer_blocks(int64_t dim, int32_t width);
CC1D_API int64_t cc1d_peer_exchange_bytes(int64_t dim, int32_t width, int32_t world);
CC1D_API int cc1d_bwd_peer_reduce(const cc1d_bwd_params* params, const cc1d_peer_reduce* peer, void* stream);

/*
 * cc1d_bwd for callers that cannot allocate device memory (a serving engine
 * that reserved almost all of HBM up front, an FFI caller without access to
 * the host framework's allocator, a loop that must not take cudaMalloc's
 * implicit synchronisation).  Identical to cc1d_bwd except that
 * params->workspace / workspace_bytes are ignored: the scratch is a static
 * device array of CC1D_NOALLOC_SCRATCH_BYTES built into the library, which
 * every GPU that loads the library holds until the process exits.  Calls
 * needing more scratch than that (see cc1d_bwd_workspace_size) fail with
 * CC1D_ERR_WORKSPACE.  The first call on a device that has something to
 * reduce looks up the array's device address on the device holding the data
 * (make it before any stream capture); calls on empty problems use no
 * scratch and make no lookup.  All calls share the array: calls that
 * overlap on the GPU race.  No allocation is made.
 * No counterpart in the reference (its backward allocates through torch).
 */
#define CC1D_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

CC1D_API int cc1d_bwd_noalloc(const cc1d_bwd_params* params, void* stream);

/*
 * Decode step of causal_conv1d_update.  x is (batch, dim, seqlen) (a 2-D x of
 * the Python API is passed with seqlen = 1).  conv_state is
 * (rows, dim, state_len) with state_len >= W-1, mutated in place:
 *   linear (cache_seqlens == NULL): shift left by seqlen, append x;
 *   circular: history read at [cache_seqlens[b]-(W-1), cache_seqlens[b]) and
 *             x written from cache_seqlens[b], both modulo state_len.
 * conv_state_indices (optional) redirects batch row b to state row
 * conv_state_indices[b]; a negative index zeroes out[b] and leaves the state
 * untouched.  cache_seqlens is always indexed by b.
 *
 * Replaces the 29-tuple built by `native_update`
 * (src/causal_conv1d_mojo/update/__init__.py:27-60).
 */
typedef struct cc1d_update_params {
  int32_t dtype;
  int32_t width;          /* 2..9 for every dtype */
  int64_t batch, dim, seqlen, state_len;
  int64_t state_rows;     /* conv_state.shape[0] (pool size when indexed) */
  int32_t silu;
  int32_t _pad0;
  const void* x;          int64_t x_batch_stride, x_dim_stride, x_seq_stride;
  const void* weight;     int64_t weight_dim_stride, weight_width_stride;
  const void* bias;       int64_t bias_stride;
  void* conv_state;       int64_t state_batch_stride, state_dim_stride, state_seq_stride;
  const int32_t* conv_state_indices; /* NULL: row b serves batch b */
  const int32_t* cache_seqlens;      /* NULL: linear mode */
  void* out;              int64_t out_batch_stride, out_dim_stride, out_seq_stride;
} cc1d_update_params;

CC1D_API int cc1d_update(const cc1d_update_params* params, void* stream);

/*
 * causal_conv1d_varlen_states: for each packed sequence i (tokens
 * [cu_seqlens[i], cu_seqlens[i+1]) of x (total_tokens, dim)), copy its last
 * state_len tokens into states[i, :, state_len-n:] and zero the rest.
 * Bit-exact data movement.
 * Replaces the Python loop of causal_conv1d_varlen_states
 * (src/causal_conv1d_mojo/causal_conv1d_varlen.py:29-61).
 */
typedef struct cc1d_varlen_states_params {
  int32_t dtype;
  int32_t _pad0;
  int64_t batch, dim, state_len, total_tokens;
  const void* x;              int64_t x_token_stride, x_dim_stride;
  const int32_t* cu_seqlens;  /* batch+1 entries, non-decreasing */
  void* states;               int64_t states_batch_stride, states_dim_stride, states_seq_stride;
} cc1d_varlen_states_params;

CC1D_API int cc1d_varlen_states(const cc1d_varlen_states_params* params, void* stream);

/*
 * The in_proj GEMM of a Mamba block with the forward conv as its epilogue
 * (bf16; widths 2..4):
 *   xBC = hidden (M, K) @ in_weight (N, K)^T, M = batch * seqlen tokens,
 *   out[m, :] = act(conv_bias + sum_j conv_weight[:, j] * xBC[m - (W-1) + j, :])
 * with the conv of cc1d_fwd applied to each sequence of seqlen tokens
 * (initial_states before its start, final_states = its last W-1 xBC rows),
 * on xBC rounded to bf16 exactly as a stored GEMM output would be.  xBC
 * itself is never written: out (M, N) is stored token-major, i.e. the
 * channel-last (batch, dim, seqlen) layout of causal_conv1d_fn.
 * Requirements: dim % 32 == 0, hidden_dim % 8 == 0, seqlen >= W-1; hidden,
 * in_weight and out with unit stride along their last dimension and
 * 16-byte aligned bases and row pitches.  Forward only.
 *
 * No counterpart in the reference: it replaces the pair "in_proj GEMM, then
 * causal_conv1d_fn" that a Mamba block runs, removing the GEMM output's
 * HBM round trip (src/causal_conv1d_mojo/_fn.py:232 allocates the conv's
 * output; fwd/kernel.mojo:161-196 reads xBC back).
 */
typedef struct cc1d_inproj_conv_params {
  int32_t dtype;            /* CC1D_BF16 */
  int32_t width;            /* 2..4 */
  int64_t batch, seqlen;
  int64_t dim;              /* N: conv channels = rows of in_weight */
  int64_t hidden_dim;       /* K */
  int32_t silu;
  int32_t _pad0;
  const void* hidden;       int64_t hidden_row_stride;      /* (M, K) */
  const void* in_weight;    int64_t in_weight_row_stride;   /* (N, K), as nn.Linear.weight */
  const void* conv_weight;  int64_t conv_weight_dim_stride, conv_weight_width_stride; /* (N, W) */
  const void* conv_bias;    int64_t conv_bias_stride;       /* NULL: no bias */
  const void* initial_states; int64_t init_batch_stride, init_dim_stride, init_seq_stride; /* NULL: zeros */
  void* out;                int64_t out_row_stride;         /* (M, N) */
  void* final_states;       int64_t final_batch_stride, final_dim_stride, final_seq_stride; /* NULL: not written */
} cc1d_inproj_conv_params;

CC1D_API int cc1d_inproj_conv_fwd(const cc1d_inproj_conv_params* params, void* stream);

/* Diagnostics: *wait_timeouts receives the number of bounded in-kernel waits
 * (pipeline barriers, peer exchanges) that gave up since the previous call,
 * and the count is reset.  The count is kept per device and this call reads
 * the CURRENT device's only: a process that drives several GPUs makes each
 * one current in turn (cudaSetDevice) and calls it once per device.  A
 * non-zero count means some results of the kernels launched meanwhile on
 * that device are invalid.  Synchronises that device.
 * No reference counterpart (the reference kernels have no in-kernel waits). */
CC1D_API int cc1d_device_status(unsigned* wait_timeouts);

/* Message of the last failed call on this thread ("" if none). */
CC1D_API const char* cc1d_last_error(void);

/* Version of the Python API this library backs ("1.6.1", as the reference's
 * __version__, src/causal_conv1d_mojo/__init__.py:51). */
CC1D_API const char* cc1d_version(void);

/* CC1D_ABI_VERSION of the loaded library. */
CC1D_API int cc1d_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CC1D_H_ */
