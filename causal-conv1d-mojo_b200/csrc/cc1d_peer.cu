// Backward dweight/dbias reduction fused with the all-reduce over the GPUs of
// a batch-sharded job, through NVLink peer memory.  sm_100a.
//
// Replaces, on every rank, the sequence finalize_kernel -> NCCL all-reduce
// of the fp32 [dweight | dbias] buffer -> casts.  The outputs are cut into
// chunks of 32; block b owns chunks b, b + grid, b + 2*grid, ...:
//   1. for each of its chunks it sums the local partial slots (as
//      finalize_kernel: 8 warps, fixed order) and pushes every sum to every
//      rank as one 8-byte word {call tag, fp32 bits}: a plain store into the
//      receiving rank's exchange buffer (this rank's row of it, in the half
//      selected by the call's parity),
//   2. polls its own exchange buffer until the words of every rank carry
//      this call's tag (bounded wait), then adds the ranks' values in rank
//      order and writes fp32 dwdb plus the parameter-dtype copies.  A wait
//      that gives up writes NaN to the outputs it could not reduce and adds
//      1 to the caller's status word (and to the process-wide counter).
// An aligned 8-byte store is seen whole or not at all, so value and tag
// travel together: no fences, no flags, no remote loads; the exchange costs
// one NVLink store latency.  The halves alternate by call parity, and a rank
// can only start call c+2 after every peer has pushed call c+1, i.e. after
// every peer has read call c -- so a word is never overwritten before it is
// read.  Every rank adds the same values in the same order, so all ranks
// hold bitwise identical gradients, reproducible run to run.
//
// The grid is capped (kPeerMaxBlocks) near what the SMs hold at once; blocks
// wait only for the blocks of the same index on other GPUs, never for blocks
// of their own GPU.  Call numbers live in device memory, one per block, so
// the kernel can be captured in a CUDA graph and replayed; all ranks must
// make the same sequence of calls.  Exchange buffers are plain device memory
// shared through CUDA IPC (no multicast objects, no TMA on peer memory).
#include <algorithm>

#include "cc1d_dispatch.cuh"

namespace cc1d {

namespace {

constexpr int kPeerWarps = 8;
constexpr i64 kPeerMaxBlocks = 1024;      // B200: 148 SMs x 8 blocks of 256 threads resident

static __device__ unsigned int g_peer_timeouts = 0;

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Rank-order sum of element e's words in this rank's buffer half `mine`
// (world words, n apart) once each carries `tag`, for the split exchange's
// FINISH, whose words have usually arrived: they are loaded 8 ranks at a
// time before any is checked, so the sum costs one memory round trip per 8
// ranks; a word that has not arrived is polled alone (bounded: false after
// max_polls polls in total).
__device__ __forceinline__ bool sum_ranks(const unsigned long long* mine, i64 n, i64 e, int world,
                                          unsigned long long tag, unsigned max_polls, float& t) {
  unsigned polls = 0;
  t = 0.f;
  for (int r0 = 0; r0 < world; r0 += 8) {
    unsigned long long v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = r0 + j < world ? ld_relaxed_sys_u64(mine + (i64)(r0 + j) * n + e) : tag;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // After a wait the rest of the batch is stale: reload before polling.
      if (polls > 0 && (v[j] & 0xffffffff00000000ull) != tag) v[j] = ld_relaxed_sys_u64(mine + (i64)(r0 + j) * n + e);
      while ((v[j] & 0xffffffff00000000ull) != tag) {
        if (++polls > max_polls) return false;
        if (polls > 64) __nanosleep(64);
        v[j] = ld_relaxed_sys_u64(mine + (i64)(r0 + j) * n + e);
      }
      if (r0 + j < world) t += __uint_as_float((unsigned)(v[j] & 0xffffffffull));
    }
  }
  return true;
}

template <typename T, int W>
__global__ void __launch_bounds__(kPeerWarps * 32) finalize_peer_kernel(const PeerFinalizeArgs p) {
  __shared__ float part[kPeerWarps][32];
  griddep_wait();  // the partials come from the backward kernel just before
  griddep_launch_dependents();
  const FinalizeArgs& a = p.f;
  const i64 n = a.D * (W + 1);
  const i64 nchunks = ceil_div(n, (i64)32);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t* ep = p.epochs + blockIdx.x;
  const uint32_t epoch = *ep + 1;  // this call's number (tag) for this block
  const unsigned long long tag = (unsigned long long)epoch << 32;
  // Word (parity, source rank, output) of a receiving rank's buffer.
  const i64 half = (i64)(epoch & 1u) * p.world * n;

  // 1. Local sums of this block's chunks, pushed to every rank.
  for (i64 ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
    const i64 e = ch * 32 + lane;
    float s = 0.f;
    if (e < n)
      for (i64 i = warp; i < a.n_partials; i += kPeerWarps) s += a.partials[i * n + e];
    part[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && e < n) {
      s = part[0][lane];
#pragma unroll
      for (int w2 = 1; w2 < kPeerWarps; ++w2) s += part[w2][lane];
      const unsigned long long word = tag | __float_as_uint(s);
      const i64 off = half + (i64)p.rank * n + e;
      for (int r = 0; r < p.world; ++r) st_relaxed_sys_u64(p.bufs[r] + off, word);
    }
    __syncthreads();
  }

  // 2. Rank-order sums of this block's chunks, one chunk per warp at a time.
  const unsigned long long* mine = p.bufs[p.rank] + half;
  for (i64 ch0 = blockIdx.x; ch0 < nchunks; ch0 += (i64)kPeerWarps * gridDim.x) {
    const i64 ch = ch0 + (i64)warp * gridDim.x;
    const i64 e = ch * 32 + lane;
    const bool active = ch < nchunks && e < n;
    bool ok = true;
    float t = 0.f;
    if (active) {
      // Polled rank by rank: here the peers' words are usually still on their
      // way (the exchange starts in this kernel), and loading them in batches
      // measured slower (C2 backward with the exchange, 8 GPUs: 112.7 -> 117.2 us).
      unsigned polls = 0;
      for (int r = 0; r < p.world && ok; ++r) {
        unsigned long long w = ld_relaxed_sys_u64(mine + (i64)r * n + e);
        while ((w & 0xffffffff00000000ull) != tag) {
          if (++polls > p.max_polls) {
            ok = false;
            break;
          }
          if (polls > 64) __nanosleep(64);
          w = ld_relaxed_sys_u64(mine + (i64)r * n + e);
        }
        t += __uint_as_float((unsigned)(w & 0xffffffffull));
      }
    }
    if (__any_sync(kFull, active && !ok) && lane == 0) {
      atomicAdd(&g_peer_timeouts, 1u);
      if (p.status != nullptr) atomicAdd(p.status, 1u);
    }
    if (!active) continue;
    // An output whose exchange timed out is written as NaN (never left
    // stale): a caller that skips the status check still sees the failure
    // in the gradients instead of silently training on garbage.
    if (!ok) t = __uint_as_float(0x7fc00000u);
    const i64 c = e / (W + 1);
    const int k = (int)(e - c * (W + 1));
    if (k < W) {
      a.dwdb[c * W + k] = t;
      if (a.dw_out) static_cast<T*>(a.dw_out)[c * a.dws_c + k * a.dws_k] = Cvt<T>::to(t);
    } else {
      if (!a.has_bias) t = 0.f;
      a.dwdb[a.D * W + c] = t;
      if (a.db_out && a.has_bias) static_cast<T*>(a.db_out)[c * a.dbs] = Cvt<T>::to(t);
    }
  }
  // Advance the call number (every thread read it above).  Counted even
  // after a timeout, so this rank's call numbers keep matching its peers'.
  __syncthreads();
  if (threadIdx.x == 0) *ep = epoch;
}

// Split exchange (CC1D_PEER_PUSH, then CC1D_PEER_FINISH): the backward's
// reduction only sums and pushes (peer_push_kernel, step 1 above), and a
// later launch -- typically on another stream, overlapping the caller's next
// work -- waits for the ranks' words and writes the outputs
// (peer_finish_kernel, step 2).  The two kernels run different grids, so
// each has one call counter for all its blocks instead of one per block:
// ctr[0] (push) and ctr[2] (finish) are read by every block at its start and
// advanced by the block that finishes last (ctr[1], ctr[3] count the
// finished blocks), which is after every block has read them.  Call c's
// FINISH must complete before the same rank's PUSH of call c+1 starts (the
// caller orders the streams): then a rank's push c+2 waited, through its
// finish c+1, for every peer's push c+1, which each peer issued after its
// own finish c -- so no word is overwritten before it is read, as above.
constexpr i64 kFinishBlocks = 1024;  // one chunk per warp: the words have usually arrived

__device__ __forceinline__ void advance_call(uint32_t* ctr, uint32_t call) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&ctr[1], 1u);
    if (prev == gridDim.x - 1) {  // every block has read ctr[0]
      ctr[1] = 0;
      ctr[0] = call;
    }
  }
}

template <typename T, int W>
__global__ void __launch_bounds__(kPeerWarps * 32) peer_push_kernel(const PeerFinalizeArgs p) {
  __shared__ float part[kPeerWarps][32];
  griddep_wait();  // the partials come from the backward kernel just before
  griddep_launch_dependents();
  const FinalizeArgs& a = p.f;
  const i64 n = a.D * (W + 1);
  const i64 nchunks = ceil_div(n, (i64)32);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t call = p.epochs[0] + 1;
  const unsigned long long tag = (unsigned long long)call << 32;
  const i64 half = (i64)(call & 1u) * p.world * n;
  for (i64 ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
    const i64 e = ch * 32 + lane;
    float s = 0.f;
    if (e < n)
      for (i64 i = warp; i < a.n_partials; i += kPeerWarps) s += a.partials[i * n + e];
    part[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && e < n) {
      s = part[0][lane];
#pragma unroll
      for (int w2 = 1; w2 < kPeerWarps; ++w2) s += part[w2][lane];
      const unsigned long long word = tag | __float_as_uint(s);
      const i64 off = half + (i64)p.rank * n + e;
      for (int r = 0; r < p.world; ++r) st_relaxed_sys_u64(p.bufs[r] + off, word);
    }
    __syncthreads();
  }
  advance_call(p.epochs, call);
}

template <typename T, int W>
__global__ void __launch_bounds__(kPeerWarps * 32) peer_finish_kernel(const PeerFinalizeArgs p) {
  griddep_wait();
  griddep_launch_dependents();
  const FinalizeArgs& a = p.f;
  const i64 n = a.D * (W + 1);
  const i64 nchunks = ceil_div(n, (i64)32);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t call = p.epochs[2] + 1;
  const unsigned long long tag = (unsigned long long)call << 32;
  const unsigned long long* mine = p.bufs[p.rank] + (i64)(call & 1u) * p.world * n;
  for (i64 ch = (i64)blockIdx.x * kPeerWarps + warp; ch < nchunks; ch += (i64)gridDim.x * kPeerWarps) {
    const i64 e = ch * 32 + lane;
    const bool active = e < n;
    bool ok = true;
    float t = 0.f;
    if (active) ok = sum_ranks(mine, n, e, p.world, tag, p.max_polls, t);
    if (__any_sync(kFull, active && !ok) && lane == 0) {
      atomicAdd(&g_peer_timeouts, 1u);
      if (p.status != nullptr) atomicAdd(p.status, 1u);
    }
    if (!active) continue;
    if (!ok) t = __uint_as_float(0x7fc00000u);  // never stale: NaN, as in the fused kernel
    const i64 c = e / (W + 1);
    const int k = (int)(e - c * (W + 1));
    if (k < W) {
      a.dwdb[c * W + k] = t;
      if (a.dw_out) static_cast<T*>(a.dw_out)[c * a.dws_c + k * a.dws_k] = Cvt<T>::to(t);
    } else {
      if (!a.has_bias) t = 0.f;
      a.dwdb[a.D * W + c] = t;
      if (a.db_out && a.has_bias) static_cast<T*>(a.db_out)[c * a.dbs] = Cvt<T>::to(t);
    }
  }
  advance_call(p.epochs + 2, call);
}

struct LaunchPeer {
  const PeerFinalizeArgs& p;
  int mode;  // 0 fused, 1 push, 2 finish
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    const dim3 block(kPeerWarps * 32);
    if (mode == 1) return launch_pdl(peer_push_kernel<T, W>, dim3((unsigned)p.nblocks), block, 0, stream, p);
    if (mode == 2) {
      const i64 nchunks = ceil_div(p.f.D * (i64)(W + 1), (i64)32);
      const i64 nb = std::min<i64>(kFinishBlocks, ceil_div(nchunks, (i64)kPeerWarps));
      return launch_pdl(peer_finish_kernel<T, W>, dim3((unsigned)nb), block, 0, stream, p);
    }
    return launch_pdl(finalize_peer_kernel<T, W>, dim3((unsigned)p.nblocks), block, 0, stream, p);
  }
};

}  // namespace

i64 peer_blocks(i64 dim, int width) {
  const i64 chunks = ceil_div(dim * (width + 1), (i64)32);
  return chunks < kPeerMaxBlocks ? chunks : kPeerMaxBlocks;
}

i64 peer_exchange_bytes(i64 dim, int width, int world) {
  return 2 * (i64)world * dim * (width + 1) * (i64)sizeof(unsigned long long);
}

cudaError_t launch_finalize_peer(int dtype, int width, const PeerFinalizeArgs& p, int mode, cudaStream_t stream) {
  if (p.nblocks <= 0) return cudaSuccess;
  return dispatch(dtype, width, LaunchPeer{p, mode, stream});
}

cudaError_t read_peer_timeouts(unsigned* count) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_peer_timeouts, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  *count += v;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_peer_timeouts, &zero, sizeof(unsigned));
}

}  // namespace cc1d
