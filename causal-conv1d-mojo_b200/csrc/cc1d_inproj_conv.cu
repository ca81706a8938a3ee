// In_proj GEMM with the causal conv as its epilogue, for sm_100a (tcgen05).
//
// In a Mamba block the conv's input is the output of the in_proj GEMM:
//   xBC[m, n] = sum_k hidden[m, k] * in_weight[n, k]        (M tokens, N channels)
//   out[m, n] = act(bias[n] + sum_j w[n, j] * xBC[m - (W-1) + j, n])
// with the taps restricted to the token's own sequence (m = b * L + t; taps at
// t - (W-1) + j < 0 read initial_states[b, n, t + j], or 0).  Run as two
// kernels, xBC makes a full HBM round trip: the GEMM writes it and the conv
// reads it back (src/causal_conv1d_mojo/_fn.py:232, the out = empty_like(x)
// the conv kernel fills, fwd/kernel.mojo:161-196 its reads).  Here the conv is
// applied to the GEMM's accumulator tile before anything leaves the SM, so
// xBC is never stored; only out (and final_states) are.
//
// Kernel: persistent, clusters of two CTAs (one per SM) computing one
// 256-token x 256-channel tile together with 2-SM MMAs (cta_group::2).
// CTA c of a pair owns the tile's 128 GEMM rows of M-tile 2*pair_m + c and
// loads them (A), plus channels [n0 + 128c, n0 + 128c + 128) of in_weight
// (its half of B); each tcgen05.mma of the pair's leader CTA reads A and B
// from both CTAs' shared memory and writes each CTA's 128 accumulator rows
// into that CTA's TMEM.  Per CTA, 6 warps:
//   warp 0      TMA producer: [128 x 64] tiles of hidden and of in_weight
//               (bf16, K-major, 128-byte swizzle) into a 6-stage ring; the
//               loads of both CTAs complete on the leader's "full" barrier.
//   warp 1      allocates 512 TMEM columns (two 128 x 256 fp32 accumulators,
//               in both CTAs); in the leader, one lane issues tcgen05.mma
//               (M=256, N=256, K=16, bf16 in, fp32 accumulate) and commits
//               each stage back to both CTAs' producers and, after the last
//               K step, the accumulator to both CTAs' epilogues.
//   warps 2..9  epilogue: each thread reads half of its TMEM lane (= tile
//               row) with tcgen05.ld, rounds it to bf16 exactly as the
//               unfused GEMM would store xBC, and writes it to a 64 KB
//               shared-memory staging tile -- the accumulator goes back to
//               the MMA issuer right then; then the roles turn: a thread
//               owns two adjacent channels and half of the rows, keeps their
//               weights, bias and W-1 previous inputs in registers and walks
//               the rows 8 at a time (loads first, then 8 independent
//               outputs) with packed fp32 math (the tap order and SiLU of
//               every other kernel of this library), each warp storing 128
//               contiguous output bytes per row, while the next tiles' MMAs
//               run.
// The two accumulators alternate, so the epilogue of one tile overlaps the
// MMAs of the next.  Per K step a CTA moves 32 KB (its A rows and half of
// B) for 128 x 256 x 64 MACs: a 128 x 256 tile on one SM moves 48 KB for
// the same work, and a 256 x 256 tile on one SM needs all of its TMEM for
// one tile (no overlap).  Measured on B200 at the Mamba-2 prefill shape
// (16384 x 2560 @ 2560 x 5376, W = 4), in the order tried: 485 us (one SM,
// 128 x 256: tensor pipe 32% busy, waiting on TMA), 461 us (one SM,
// 256 x 256), 433 us (this pairing, row-per-thread epilogue), ~350 us
// (channel-pair walk, whole accumulator staged before the walk).  Without
// the conv walk the same kernel runs the GEMM in ~308 us, as fast as cuBLAS
// (~300-305 us); the walk alone takes ~6.7 us per tile, less than a tile's
// MMAs (~16 us), so its remaining cost is contention, not serialisation.

// Halo: the conv of output row m needs xBC rows m-(W-1) .. m.  A CTA's 128
// GEMM rows start W-1 rows before its first output row, so each carries its
// own halo and produces 128-(W-1) output rows (2.4% extra MMA work at
// W = 4).  The first W-1 rows are computed but not stored.  No TMA load in
// this file uses cluster multicast; the leader reaches its peer's barriers
// through mapa addresses.
//
// Every mbarrier wait is bounded; a wait that gives up sets a block-wide
// abort flag, every role stops issuing, waits (bounded) for the copies and
// MMAs it already issued, and the TMEM is released before the block exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

#include "cc1d.h"
#include "cc1d_dispatch.cuh"
#include "cc1d_tma.cuh"

namespace cc1d {

namespace {

constexpr int kBM = 128;       // GEMM rows per tile (tokens, halo included)
constexpr int kBN = 256;       // channels per tile
constexpr int kBK = 64;        // K per stage: 64 bf16 = one 128-byte swizzle row
#ifndef CC1D_INPROJ_STAGES
#define CC1D_INPROJ_STAGES 4
#endif
constexpr int kStages = CC1D_INPROJ_STAGES;
constexpr int kUmmaK = 16;     // K per tcgen05.mma (kind::f16)
constexpr int kChunk = kBN;    // the whole accumulator row is staged at once
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr unsigned kABytes = kBM * kBK * 2;     // 16 KB
constexpr unsigned kBBytes = (kBN / 2) * kBK * 2;  // 16 KB: this CTA's half of B
constexpr unsigned kStageBytes = kABytes + kBBytes;
constexpr int kYPitch = kChunk * 2;             // bytes per staged row; 16-byte units XOR-swizzled by row
constexpr unsigned kYBytes = kBM * kYPitch;     // the staged chunk (bf16)
constexpr int kTmemCols = 2 * kBN;              // two accumulators (in each CTA of the pair)

// Shared-memory map (offsets from a 1024-byte aligned base).
constexpr unsigned kOffA = 0;
constexpr unsigned kOffB = kOffA + kStages * kABytes;
constexpr unsigned kOffY = kOffB + kStages * kBBytes;
constexpr unsigned kPairStageBytes = 2 * kStageBytes;           // both CTAs' loads of one stage
constexpr unsigned kOffBar = kOffY + kYBytes;
constexpr unsigned kSmemBytes = kOffBar + 256 + 1024;           // barriers, TMEM slot, alignment slack
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a block may use");

static_assert(kOffB % 1024 == 0 && kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzled tiles need 1 KB alignment");

struct alignas(64) FusedParams {
  CUtensorMap map_a;   // hidden (M, K)
  CUtensorMap map_b;   // in_weight (N, K)
  const __nv_bfloat16* cw; i64 cw_c, cw_k;
  const __nv_bfloat16* bias; i64 bs;
  const __nv_bfloat16* init; i64 is_b, is_c, is_l;
  __nv_bfloat16* out; i64 os_m;
  __nv_bfloat16* fin; i64 fs_b, fs_c, fs_l;
  i64 B, L, M, N, K;
  int silu;
  int m_tiles, n_tiles, k_blocks, out_rows;
  unsigned* abort_count;  // device counter of blocks that gave up (diagnostics)
};

// ---- tcgen05 / TMEM primitives (inline PTX) ----

// TMEM of a CTA pair: the warp of the same index in both CTAs allocates
// (and later frees) the same columns in both CTAs' TMEM.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, int cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank`
// of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// All threads of both CTAs (release / acquire: barrier inits, TMEM state).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded wait, with cluster-scope acquire, for a phase of a barrier that
// the other CTA of the pair arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < kSpinLimit; ++i) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  atomicAdd(&g_cc1d_wait_timeouts, 1u);
  return false;
}

// Arrive on an mbarrier given by its shared::cluster address (either CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrives once on the mbarrier at shared::cluster address `bar` (in either
// CTA of the pair) when every 2-SM tcgen05.mma this thread issued before has
// completed (its shared-memory operands read, its accumulators written).
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 2-SM MMA, issued by the leader CTA: D (256 x N, rows 0..127 in the
// leader's TMEM, 128..255 in the peer's) (+)= A (rows 0..127 from the
// leader's shared memory, 128..255 from the peer's, same address) * B^T
// (N/2 rows from each CTA), both K-major.
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major bf16 tile stored with the
// 128-byte swizzle (rows of 64 elements, 8-row groups 1024 bytes apart):
// start address >> 4, leading byte offset 16 (unused by this layout),
// stride byte offset 1024, descriptor version 1, swizzle mode 2 (128 B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, N = kBN, M = 2 * kBM (the pair's rows).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)((2 * kBM) >> 4) << 24);

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on the mbarrier at shared::cluster address `bar` (the pair leader's).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Named barrier of the epilogue warps (non-aligned form: correct even if
// the compiler left the warps' lanes diverged at this point).
__device__ __forceinline__ void epi_bar() { asm volatile("barrier.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

// The same barrier, returning to every epilogue thread the OR of `pred`
// over all of them (one decision taken by all).
__device__ __forceinline__ bool epi_bar_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kEpiWarps * 32)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ bool aborted(volatile int* flag) { return *flag != 0; }

template <int W, bool SILU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    inproj_conv_kernel(const __grid_constant__ FusedParams p) {
  constexpr int H = W - 1;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);  // leader: both CTAs' loads of a stage
  uint64_t* empty = full + kStages;                               // each CTA: its stage may be refilled
  uint64_t* tfull = empty + kStages;                              // each CTA: accumulator ready
  uint64_t* tempty = tfull + 2;                                   // leader: both epilogues drained it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();  // 0: leader (issues the MMAs), 1: peer
  const bool leader = crank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_tiles = p.m_tiles * p.n_tiles;  // pair tiles: (M-tile pair, channel tile)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      prefetch_tensormap(&p.map_a);
      prefetch_tensormap(&p.map_b);
      unsigned k = 0;
      for (int tile = pair; tile < num_tiles && !aborted(abort_flag); tile += npairs) {
        const int nt = tile % p.n_tiles, mp = tile / p.n_tiles;
        const int row0 = (2 * mp + (int)crank) * p.out_rows - H;  // this CTA's first GEMM row (halo)
        const int brow0 = nt * kBN + (int)crank * (kBN / 2);       // this CTA's half of the channel tile
        for (int kb = 0; kb < p.k_blocks; ++kb, ++k) {
          const unsigned s = k % kStages, use = k / kStages;
          if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], kPairStageBytes);
          const uint32_t fb = peer_addr(&full[s], 0);
          tma_load_2d(smem + kOffA + s * kABytes, &p.map_a, fb, kb * kBK, row0);
          tma_load_2d(smem + kOffB + s * kBBytes, &p.map_b, fb, kb * kBK, brow0);
        }
      }
      // The leader waits for the last stages of both CTAs (they complete on
      // its barriers); the peer's in-flight loads are covered by that wait,
      // which precedes the cluster barrier both CTAs meet before exiting.
      if (leader) mbar_drain(full, k, kStages);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (lane == 0 && leader) {
      unsigned k = 0, j = 0;
      uint64_t* last = nullptr;
      unsigned last_parity = 0;
      for (int tile = pair; tile < num_tiles && !aborted(abort_flag); tile += npairs, ++j) {
        const unsigned acc = j & 1, use = j >> 1;
        // Both CTAs' epilogues must have drained this accumulator (first two tiles: free).
        if (!mbar_wait_cluster(&tempty[acc], (use & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kBN;
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++k) {
          const unsigned s = k % kStages, u = k / kStages;
          if (!mbar_wait(&full[s], u & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + kOffA + s * kABytes);
          const uint32_t b0 = smem_u32(smem + kOffB + s * kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            tc_mma(d, sw128_desc(a0 + kk * kUmmaK * 2), sw128_desc(b0 + kk * kUmmaK * 2), kIdesc,
                   (kb | kk) != 0 ? 1u : 0u);
          // Both CTAs' stage s is free once these MMAs have read it.
          tc_commit(peer_addr(&empty[s], 0));
          tc_commit(peer_addr(&empty[s], 1));
          last = &empty[s];
          last_parity = u & 1;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        tc_commit(peer_addr(&tfull[acc], 0));  // accumulator complete, in both CTAs
        tc_commit(peer_addr(&tfull[acc], 1));
      }
      // Keep the pair (and its TMEM) until the MMAs issued last are done.
      if (last != nullptr) (void)mbar_wait(last, last_parity);
    }
  } else {
    // ---------------- epilogue (both CTAs) ----------------
    const int ew = warp - 2;                // 0..7
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int hc = ew >> 2;                 // which 128 channels of the tile it stages
    const int r_own = q * 32 + lane;        // tile row this thread stages (= TMEM lane)
    const int et = threadIdx.x - 64;        // 0..255
    const int cp = et & 127;                // channel pair of the tile this thread walks
    const int rg = et >> 7;                 // rows it stores: [64 rg, 64 rg + 64)
    const uint32_t tempty_leader = peer_addr(tempty, 0);
    typedef Pair<__nv_bfloat16> P;
    unsigned j = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs, ++j) {
      const int nt = tile % p.n_tiles, mp = tile / p.n_tiles;
      const int col0 = nt * kBN;
      const i64 mrow0 = (i64)(2 * mp + (int)crank) * p.out_rows - H;  // token of tile row 0
      // Conv weights and bias of this thread's channel pair, fetched before
      // waiting for the accumulator so that their latency overlaps the MMAs.
      const i64 n = col0 + 2 * cp;
      const bool nv = n < p.N;
      float2 wv[W];
#pragma unroll
      for (int kk = 0; kk < W; ++kk)
        wv[kk] = nv ? f2(__bfloat162float(p.cw[n * p.cw_c + kk * p.cw_k]),
                         __bfloat162float(p.cw[(n + 1) * p.cw_c + kk * p.cw_k]))
                    : f2(0.f, 0.f);
      const float2 bv = (nv && p.bias) ? f2(__bfloat162float(p.bias[n * p.bs]), __bfloat162float(p.bias[(n + 1) * p.bs]))
                                       : f2(0.f, 0.f);
      const unsigned acc = j & 1, use = j >> 1;
      const bool ok = mbar_wait(&tfull[acc], use & 1);
      if (!ok) *abort_flag = 1;
      // One decision for all epilogue threads (so that their barriers keep
      // matching): stop if any of them timed out or another role aborted.
      if (epi_bar_or(!ok || aborted(abort_flag))) break;
      tc_fence_after();
      // 1. Stage: 128 channels of this thread's row, bf16-rounded.  16-byte
      //    unit u of row r sits at unit u ^ (r & 7): rows 128 bytes apart hit
      //    the same banks, so the XOR spreads both the row-wise stores (8
      //    rows per phase) and the column-wise loads of the walk.
      {
        uint4* yrow = reinterpret_cast<uint4*>(smem + kOffY + r_own * kYPitch);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t v[32];
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * kBN + hc * 128 + g * 32, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = P::pack(f2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int u = hc * 16 + g * 4 + i;  // 16-byte unit (8 channels) of the row
            yrow[u ^ (r_own & 7)] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          }
        }
        // Accumulator fully read: hand it back to the leader's MMA issuer.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader + acc * 8);
      }
      epi_bar();
      // 2. Walk: channels (n, n+1); rows [64 rg - 8, 64 rg + 64) of the tile,
      //    the first 8 (rg > 0) only filling the W-1 window.  The next
      //    tile's staging waits at its opening barrier for every walk to end.
      if (nv) {
        const int r0 = rg == 0 ? 0 : 64 * rg - 8;   // first row walked
        const int rs = rg == 0 ? H : 64 * rg;        // first row stored
        i64 m = mrow0 + r0;
        // Sequence position of the first walked row (one division per walk);
        // rows before token 0 (the first tile's halo) count up to t = 0.
        i64 b = m >= 0 ? m / p.L : 0;
        i64 t = m >= 0 ? m - b * p.L : m;
        float2 xw[H];
#pragma unroll
        for (int jj = 0; jj < H; ++jj) xw[jj] = f2(0.f, 0.f);
        const uint32_t* ybase = reinterpret_cast<const uint32_t*>(smem + kOffY);
        const int cu = cp >> 2, cw4 = cp & 3;  // 16-byte unit and word of this channel pair
        for (int r = r0; r < 64 * rg + 64; r += 8, m += 8) {
          uint32_t wd[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)  // r is a multiple of 8: row r + i has (r + i) & 7 == i
            wd[i] = ybase[(r + i) * (kYPitch / 4) + ((cu ^ i) << 2) + cw4];
          // Clean block: 8 rows of one sequence, none its first token, none
          // among its last W-1 (final_states), all in range and stored.
          const bool clean = r >= rs && m >= 0 && m + 8 <= p.M && t >= 1 && t + 8 <= p.L - H;
          if (clean) {
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 xv = P::unpack(wd[i]);
              float2 a2 = bv;
#pragma unroll
              for (int jj = 0; jj < H; ++jj) a2 = fma2(wv[jj], xw[jj], a2);
              a2 = fma2(wv[H], xv, a2);
              if (SILU) a2 = silu2(a2);
              o[i] = P::pack(a2);
#pragma unroll
              for (int jj = 0; jj < H - 1; ++jj) xw[jj] = xw[jj + 1];
              xw[H - 1] = xv;
            }
            __nv_bfloat16* dst = p.out + m * p.os_m + n;
#pragma unroll
            for (int i = 0; i < 8; ++i) *reinterpret_cast<uint32_t*>(dst + i * p.os_m) = o[i];
            t += 8;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i, ++t) {
              const i64 mi = m + i;
              if (t == p.L) {  // next sequence
                t = 0;
                ++b;
              }
              if (mi >= 0 && t == 0) {
                // Sequence start: the window is initial_states[b] (or zeros).
#pragma unroll
                for (int jj = 0; jj < H; ++jj)
                  xw[jj] = p.init ? f2(__bfloat162float(p.init[b * p.is_b + n * p.is_c + jj * p.is_l]),
                                       __bfloat162float(p.init[b * p.is_b + (n + 1) * p.is_c + jj * p.is_l]))
                                  : f2(0.f, 0.f);
              }
              const float2 xv = P::unpack(wd[i]);
              if (r + i >= rs && mi >= 0 && mi < p.M) {
                float2 a2 = bv;
#pragma unroll
                for (int jj = 0; jj < H; ++jj) a2 = fma2(wv[jj], xw[jj], a2);
                a2 = fma2(wv[H], xv, a2);
                if (SILU) a2 = silu2(a2);
                *reinterpret_cast<uint32_t*>(p.out + mi * p.os_m + n) = P::pack(a2);
                // final_states: xBC of the last W-1 tokens of the sequence.
                if (p.fin && t >= p.L - H) {
                  __nv_bfloat16* f = p.fin + b * p.fs_b + n * p.fs_c + (t - (p.L - H)) * p.fs_l;
                  f[0] = __ushort_as_bfloat16((unsigned short)(wd[i] & 0xffffu));
                  f[p.fs_c] = __ushort_as_bfloat16((unsigned short)(wd[i] >> 16));
                }
              }
#pragma unroll
              for (int jj = 0; jj < H - 1; ++jj) xw[jj] = xw[jj + 1];
              xw[H - 1] = xv;
            }
          }
        }
      }
    }
  }

  // Teardown: every role of both CTAs has stopped (lanes 1..31 of the
  // producer and MMA warps wait here for their lane 0); then both CTAs'
  // warp 1 release the pair's TMEM.
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (threadIdx.x == 0 && *abort_flag && p.abort_count) atomicAdd(p.abort_count, 1u);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---- host side ----

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || f == nullptr)
      return nullptr;
    fn.store(f, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// 2-D bf16 map over a row-major (rows, cols) matrix, box (64 cols, box_rows),
// 128-byte swizzle, zero fill outside.
bool make_kmajor_map(CUtensorMap* m, const void* base, i64 rows, i64 cols, i64 row_stride, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) set_error_detail("cuTensorMapEncodeTiled returned %d", (int)r);
  return r == CUDA_SUCCESS;
}

static __device__ unsigned g_fused_aborts = 0;

template <int W, bool SILU>
cudaError_t launch_fused(const FusedParams& prm, int grid, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
  if (bit == 0 || !(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(inproj_conv_kernel<W, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  inproj_conv_kernel<W, SILU><<<grid, kThreads, kSmemBytes, stream>>>(prm);  // cluster dims (2, 1, 1)
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

cudaError_t read_fused_aborts(unsigned* count) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_fused_aborts, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  *count += v;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_fused_aborts, &zero, sizeof(unsigned));
}

}  // namespace cc1d

using namespace cc1d;

extern "C" int cc1d_inproj_conv_fwd(const cc1d_inproj_conv_params* q, void* stream) {
  if (q == nullptr) return report_error(CC1D_ERR_INVALID_ARGUMENT, "cc1d_inproj_conv_fwd: params is NULL");
  if (q->dtype != CC1D_BF16)
    return report_error(CC1D_ERR_UNSUPPORTED, "cc1d_inproj_conv_fwd: only bf16 is supported (dtype code %d)", q->dtype);
  if (q->width < 2 || q->width > 4)
    return report_error(CC1D_ERR_UNSUPPORTED, "cc1d_inproj_conv_fwd: width must be in 2..4 (got %d)", q->width);
  if (q->batch < 0 || q->seqlen < 0 || q->dim < 0 || q->hidden_dim < 0)
    return report_error(CC1D_ERR_INVALID_ARGUMENT, "cc1d_inproj_conv_fwd: negative shape");
  const i64 M = q->batch * q->seqlen, N = q->dim, K = q->hidden_dim;
  if (M == 0 || N == 0) return CC1D_OK;
  if (q->seqlen < q->width - 1)
    return report_error(CC1D_ERR_UNSUPPORTED, "cc1d_inproj_conv_fwd: seqlen must be >= width-1");
  if (K == 0 || K % 8 != 0 || N % 32 != 0)
    return report_error(CC1D_ERR_UNSUPPORTED,
                        "cc1d_inproj_conv_fwd: hidden_dim must be a positive multiple of 8 and dim a multiple of 32");
  if (!q->hidden || !q->in_weight || !q->conv_weight || !q->out)
    return report_error(CC1D_ERR_INVALID_ARGUMENT, "cc1d_inproj_conv_fwd: hidden, in_weight, conv_weight, out required");
  if (!aligned16(q->hidden) || !aligned16(q->in_weight) || !aligned16(q->out) || (q->hidden_row_stride * 2) % 16 ||
      (q->in_weight_row_stride * 2) % 16 || (q->out_row_stride * 2) % 16 || q->hidden_row_stride < K ||
      q->in_weight_row_stride < K || q->out_row_stride < N)
    return report_error(CC1D_ERR_INVALID_ARGUMENT,
                        "cc1d_inproj_conv_fwd: hidden / in_weight / out need 16-byte aligned bases and row pitches "
                        "and unit stride along their last dimension");
  if (M > 0x7fffff00LL || N > 0x7fffff00LL || K > 0x7fffff00LL)
    return report_error(CC1D_ERR_UNSUPPORTED, "cc1d_inproj_conv_fwd: dimensions must fit 31 bits");
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, q->out) == cudaSuccess && at.type == cudaMemoryTypeDevice && at.device >= 0) {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != at.device) {
      cudaError_t e = cudaSetDevice(at.device);
      if (e != cudaSuccess) return report_cuda_error(e, "cc1d_inproj_conv_fwd: cudaSetDevice");
    }
  } else {
    (void)cudaGetLastError();
  }
  FusedParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!make_kmajor_map(&prm.map_a, q->hidden, M, K, q->hidden_row_stride, kBM) ||
      !make_kmajor_map(&prm.map_b, q->in_weight, N, K, q->in_weight_row_stride, kBN / 2))
    return report_cuda_error(cudaErrorInvalidValue, "cc1d_inproj_conv_fwd: tensor map");
  prm.cw = static_cast<const __nv_bfloat16*>(q->conv_weight);
  prm.cw_c = q->conv_weight_dim_stride;
  prm.cw_k = q->conv_weight_width_stride;
  prm.bias = static_cast<const __nv_bfloat16*>(q->conv_bias);
  prm.bs = q->conv_bias_stride;
  prm.init = static_cast<const __nv_bfloat16*>(q->initial_states);
  prm.is_b = q->init_batch_stride;
  prm.is_c = q->init_dim_stride;
  prm.is_l = q->init_seq_stride;
  prm.out = static_cast<__nv_bfloat16*>(q->out);
  prm.os_m = q->out_row_stride;
  prm.fin = static_cast<__nv_bfloat16*>(q->final_states);
  prm.fs_b = q->final_batch_stride;
  prm.fs_c = q->final_dim_stride;
  prm.fs_l = q->final_seq_stride;
  prm.B = q->batch;
  prm.L = q->seqlen;
  prm.M = M;
  prm.N = N;
  prm.K = K;
  prm.silu = q->silu ? 1 : 0;
  prm.out_rows = kBM - (q->width - 1);
  prm.m_tiles = (int)ceil_div(ceil_div(M, (i64)prm.out_rows), (i64)2);  // pairs of 128-row M tiles
  prm.n_tiles = (int)ceil_div(N, (i64)kBN);
  prm.k_blocks = (int)ceil_div(K, (i64)kBK);
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&prm.abort_count), g_fused_aborts);
  if (e != cudaSuccess) return report_cuda_error(e, "cc1d_inproj_conv_fwd: cudaGetSymbolAddress");
  DeviceInfo dev;
  e = device_info(&dev);
  if (e != cudaSuccess) return report_cuda_error(e, "cc1d_inproj_conv_fwd: device attributes");
  const i64 tiles = (i64)prm.m_tiles * prm.n_tiles;
  const int grid = 2 * (int)std::min<i64>(tiles, dev.sms / 2);  // CTA pairs
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool silu = q->silu != 0;
  switch (q->width) {
    case 2: e = silu ? launch_fused<2, true>(prm, grid, s) : launch_fused<2, false>(prm, grid, s); break;
    case 3: e = silu ? launch_fused<3, true>(prm, grid, s) : launch_fused<3, false>(prm, grid, s); break;
    default: e = silu ? launch_fused<4, true>(prm, grid, s) : launch_fused<4, false>(prm, grid, s); break;
  }
  if (e != cudaSuccess) return report_cuda_error(e, "cc1d_inproj_conv_fwd launch");
  return CC1D_OK;
}
