// Backward dweight/dbias reduction fused with the all-reduce over the GPUs of
// a batch-sharded job, through NVLink peer memory.  sm_100a.
//
// Replaces, on every rank, the sequence finalize_kernel -> NCCL all-reduce
// of the fp32 [dweight | dbias] buffer -> casts.  The outputs are cut into
// chunks of 32; block b owns chunks b, b + grid, b + 2*grid, ...:
//   1. for each of its chunks it sums the local partial slots (as
//      finalize_kernel: 8 warps, fixed order) and writes the 32 sums into
//      this rank's exchange buffer (peer-visible, double-buffered by call
//      parity),
//   2. publishes its flag to every rank (st.release.sys into the peer's flag
//      array) and waits until block b of every rank has published
//      (ld.acquire.sys; bounded wait),
//   3. adds the ranks' sums of its chunks in rank order (loads from peer
//      memory) and writes fp32 dwdb plus the parameter-dtype copies.
// Every rank adds the same values in the same order, so all ranks hold
// bitwise identical gradients, reproducible run to run.  The grid is capped
// (kPeerMaxBlocks) far below what the SMs hold at once, so every block of
// every rank is resident and the cross-GPU waits cannot starve; blocks never
// wait for other blocks of their own GPU.  Call numbers ("epochs") live in
// device memory, one per block, so the kernel can be captured in a CUDA
// graph and replayed; all ranks must make the same sequence of calls.  The
// exchange buffers and flags are plain device memory shared through CUDA
// IPC (no multicast objects, no TMA on peer memory).
#include "cc1d_dispatch.cuh"

namespace cc1d {

namespace {

constexpr int kPeerWarps = 8;
constexpr i64 kPeerMaxBlocks = 256;      // <= 2 blocks per SM of a B200
constexpr unsigned kPeerSpin = 1u << 22;  // polls (with back-off) before giving up

static __device__ unsigned int g_peer_timeouts = 0;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T, int W>
__global__ void __launch_bounds__(kPeerWarps * 32) finalize_peer_kernel(const PeerFinalizeArgs p) {
  __shared__ float part[kPeerWarps][32];
  __shared__ int all_arrived;
  const FinalizeArgs& a = p.f;
  const i64 n = a.D * (W + 1);
  const i64 nchunks = ceil_div(n, (i64)32);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint32_t* ep = p.epochs + blockIdx.x;
  const uint32_t epoch = *ep + 1;  // this call's number for this block
  const i64 parity_off = (i64)(epoch & 1u) * n;
  float* mine = p.bufs[p.rank] + parity_off;

  // 1. Local sums of this block's chunks into the exchange buffer.
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
      mine[e] = s;
    }
    __syncthreads();
  }

  // 2. Publish, then wait for block blockIdx.x of every rank.
  if (warp == 0) {
    __threadfence_system();
    __syncwarp();
    if (lane < p.world) st_release_sys(p.flags[lane] + (i64)p.rank * p.nblocks + blockIdx.x, epoch);
    bool ok = true;
    if (lane < p.world) {
      const uint32_t* f = p.flags[p.rank] + (i64)lane * p.nblocks + blockIdx.x;
      unsigned i = 0;
      while (ld_acquire_sys(f) < epoch) {
        if (++i > kPeerSpin) {
          ok = false;
          break;
        }
        if (i > 32) __nanosleep(128);
      }
    }
    ok = __all_sync(kFull, ok);
    if (lane == 0) {
      all_arrived = ok ? 1 : 0;
      if (!ok) atomicAdd(&g_peer_timeouts, 1u);
      // Counted even after a timeout, so this rank's call numbers keep
      // matching its peers'.
      *ep = epoch;
    }
  }
  __syncthreads();
  if (!all_arrived) return;  // outputs stay unwritten; the host reads the count
  // Every thread acquires every rank's flag itself (all already set), so its
  // peer loads are ordered after each peer's release.
  for (int r = 0; r < p.world; ++r) (void)ld_acquire_sys(p.flags[p.rank] + (i64)r * p.nblocks + blockIdx.x);

  // 3. Rank-order sums of this block's chunks, one chunk per warp at a time.
  for (i64 ch = blockIdx.x + (i64)warp * gridDim.x; ch < nchunks; ch += (i64)kPeerWarps * gridDim.x) {
    const i64 e = ch * 32 + lane;
    if (e >= n) continue;
    float t = 0.f;
    for (int r = 0; r < p.world; ++r) t += __ldcv(p.bufs[r] + parity_off + e);
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
}

struct LaunchPeer {
  const PeerFinalizeArgs& p;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    finalize_peer_kernel<T, W><<<(unsigned)p.nblocks, kPeerWarps * 32, 0, stream>>>(p);
    return cudaGetLastError();
  }
};

}  // namespace

i64 peer_blocks(i64 dim, int width) {
  const i64 chunks = ceil_div(dim * (width + 1), (i64)32);
  return chunks < kPeerMaxBlocks ? chunks : kPeerMaxBlocks;
}

cudaError_t launch_finalize_peer(int dtype, int width, const PeerFinalizeArgs& p, cudaStream_t stream) {
  if (p.nblocks <= 0) return cudaSuccess;
  return dispatch(dtype, width, LaunchPeer{p, stream});
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
