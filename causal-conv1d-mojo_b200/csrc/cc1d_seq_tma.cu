// seqlen-contiguous (x.stride(2) == 1) forward and backward kernels, fed by a
// TMA pipeline.  sm_100a.
//
// Block = 4 consumer warps + 1 producer warp, owning a group of 8 channels of
// one batch row and a segment of positions.  The producer's elected lane
// streams [8 channel-rows x 256 positions] tiles (cp.async.bulk.tensor.3d over
// the (L, D, B) view) into a shared-memory ring guarded by full/empty
// mbarriers (bounded waits).  Consumer warp w owns channel rows 2w and 2w+1:
// lane i holds positions [8i, 8i+8) of both rows, packed as (row 2w, row 2w+1)
// float2 pairs so the conv taps run as sm_100 FFMA2; the W-1 halo of lane i
// comes from lane i-1 by shuffle, and lane 0 of the next tile takes it from
// lane 31 of the current one, so x is read from HBM exactly once.
//
// The backward walks the tiles forward too.  dx at a position needs dpre of
// the next W-1 positions; its tiles overlap by one lane (they advance 248
// positions), so lane 31 recomputes the dpre lane 30's dx needs and every
// tile's dx is emitted within the tile.  (The shifted-row backward instead
// emits each tile's dx one tile late.)
// Semantics are those of cc1d_fwd.cu / cc1d_bwd.cu (reference CPU kernels
// src/causal_conv1d_mojo/fwd_cpu/kernel.mojo:64-117,
// bwd_full_cpu/kernel.mojo:26-314; final/initial states as
// src/causal_conv1d_mojo/reference.py:50-56).
//
// Rows whose pitch is not a multiple of 16 bytes (odd lengths of contiguous
// tensors) take the "shifted" kernels below, which stream the same tiles
// through a 2-D view of the tensor laid on its own 16-byte grid.
#include <cudaTypedefs.h>

#include <type_traits>

#include "cc1d_dispatch.cuh"
#include "cc1d_tma.cuh"

namespace cc1d {

namespace {

// Tunables (measured on B200; overridable at build time for sweeps).
#ifndef CC1D_SEQ_WARPS
#define CC1D_SEQ_WARPS 4        // consumer warps per block
#endif
#ifndef CC1D_SEQ_FWD_STAGES16
#define CC1D_SEQ_FWD_STAGES16 8  // forward ring stages, 16-bit types
#endif
#ifndef CC1D_SEQ_FWD_STAGES32
#define CC1D_SEQ_FWD_STAGES32 4  // forward ring stages, fp32
#endif
#ifndef CC1D_SEQ_BWD_STAGES16
#define CC1D_SEQ_BWD_STAGES16 4  // backward ring stages (x + dout tiles), 16-bit types
#endif
#ifndef CC1D_SEQ_BWD_STAGES32
#define CC1D_SEQ_BWD_STAGES32 3  // backward ring stages, fp32
#endif
#ifndef CC1D_SEQ_FWD_MIN_BLOCKS
#define CC1D_SEQ_FWD_MIN_BLOCKS 1
#endif
#ifndef CC1D_SEQ_FWD_FAST_MIN_BLOCKS
#define CC1D_SEQ_FWD_FAST_MIN_BLOCKS 5  // 16-bit, no seq_idx, W <= 7: <= 72 registers without spills
                                        // (B200: C5 W=4 SiLU fwd 706 -> 659 us, L=2048 rows 74 -> 66 us)
#endif
#ifndef CC1D_SEQ_BWD_MIN_BLOCKS
#define CC1D_SEQ_BWD_MIN_BLOCKS 4  // widths <= 5: registers capped at 96, 4 blocks per SM (3 without: -16% at C5)
#endif
#ifndef CC1D_SEQ_BWD_IDS_MIN_BLOCKS
#define CC1D_SEQ_BWD_IDS_MIN_BLOCKS 3  // with seq_idx (4 fits W <= 4 in 96 registers but measured 2% slower)
#endif
#ifndef CC1D_SEQ_FWD_SH_MIN_BLOCKS
#define CC1D_SEQ_FWD_SH_MIN_BLOCKS 5  // shifted rows: <= 80 registers, 5 blocks per SM (the smem limit)
#endif
#ifndef CC1D_SEQ_BWD_SH_MIN_BLOCKS
#define CC1D_SEQ_BWD_SH_MIN_BLOCKS 4  // shifted rows (overlapping tiles: 8 bytes of spills at W = 4)
#endif

constexpr int kSW = CC1D_SEQ_WARPS;  // consumer warps
constexpr int kRows = 2 * kSW;       // channel rows per tile
constexpr int kTL = 256;             // positions per tile (32 lanes x 8)
constexpr int kThreadsSeq = (kSW + 1) * 32;
constexpr int kBwdStep = kTL - 8;    // backward tiles advance by 31 lanes (see bwd_seq_tma_kernel)

template <typename T>
constexpr unsigned seq_tile_bytes() {
  return kTL * kRows * sizeof(T);
}
template <typename T>
constexpr int seq_fwd_stages() {
  return sizeof(T) == 2 ? CC1D_SEQ_FWD_STAGES16 : CC1D_SEQ_FWD_STAGES32;
}
template <typename T>
constexpr int seq_bwd_stages() {
  return sizeof(T) == 2 ? CC1D_SEQ_BWD_STAGES16 : CC1D_SEQ_BWD_STAGES32;
}

// Bytes of a stage's sequence-id tile (kTL int32 ids), present with seq_idx.
constexpr unsigned kIdsBytes = kTL * sizeof(int);

// Sequence masks (backward with seq_idx).  seq_mask_kernel runs first and
// writes one uint16 per position q of each batch row: bit j (j < W-1) set
// when position q-1-j exists and carries q's sequence id, bit 15 when q's id
// is >= 0 (not padding).  A tap of the conv (or of its transpose) between
// two positions counts exactly when the later position's mask has the bit of
// their distance, so the backward reads one 16-byte mask vector per lane and
// tile instead of ids and their halos, and a tile whose masks are all full
// takes the ungated path.  Row pitch: L rounded up to 8 positions.
constexpr unsigned kMaskBytes = kTL * sizeof(uint16_t);
constexpr uint32_t kMaskValid = 0x8000u;
template <int H>
constexpr uint32_t mask_full() {
  return ((1u << H) - 1u) | kMaskValid;
}
__host__ __device__ inline i64 mask_pitch(i64 L) { return (L + 7) / 8 * 8; }

__global__ void __launch_bounds__(256) seq_mask_kernel(const int* __restrict__ seq, i64 ss_b, i64 ss_l, i64 B,
                                                       i64 L, int H, uint16_t* __restrict__ mask) {
  griddep_wait();  // seq_idx may come from the previous kernel; the mask buffer may still be read by it
  griddep_launch_dependents();
  const i64 Lp = mask_pitch(L);
  const i64 q = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= Lp) return;
  for (i64 b = blockIdx.y; b < B; b += gridDim.y) {
    uint32_t m = 0;
    if (q < L) {
      const int* sb = seq + b * ss_b;
      const int id = sb[q * ss_l];
      m = id >= 0 ? kMaskValid : 0u;
      for (int j = 0; j < H; ++j) {
        const i64 r = q - 1 - j;
        if (r >= 0 && sb[r * ss_l] == id) m |= 1u << j;
      }
    }
    mask[b * Lp + q] = (uint16_t)m;
  }
}

// The 8 masks of a lane's positions as 4 words (position 2k in the low half
// of word k), and the mask of position i (i < 8 compile-time).
__device__ __forceinline__ void lds_masks(const unsigned char* tile, int lane, uint32_t (&m)[4]) {
  const uint4 u = *reinterpret_cast<const uint4*>(tile + lane * 16);
  m[0] = u.x; m[1] = u.y; m[2] = u.z; m[3] = u.w;
}
__device__ __forceinline__ uint32_t mask_at(const uint32_t (&m)[4], int i) {
  return (m[i >> 1] >> (16 * (i & 1))) & 0xffffu;
}

// Shifted-row geometry (rows whose pitch is not a multiple of 16 bytes):
// the tensor viewed as rows of `in` elements; a row tile is one box of
// `rows` such rows starting at the one that holds the tile's first element.
struct ShiftGeom {
  int in;        // elements per view row (a power of two, 16..128 bytes)
  int in_log2;
  int rows;      // kTL / in + 1
  unsigned tx;   // bytes one tensor's tile delivers (kRows boxes)
  // Tiles of a segment: seg_len / step (step = the positions a tile
  // advances: kTL forward, kBwdStep backward), and for a row's last segment
  // enough to reach L from its start - (E - 1).  Counted on the host.
  int tiles_full, tiles_last;
};

struct alignas(64) SeqFwdParams {
  CUtensorMap map_x;
  CUtensorMap map_s;  // seq_idx as (L, 1, B) int32, when given
  FwdArgs a;
  i64 groups;
  ShiftGeom sg;
};
struct alignas(64) SeqBwdParams {
  CUtensorMap map_x;
  CUtensorMap map_g;
  CUtensorMap map_s;
  BwdArgs a;
  i64 groups;
  ShiftGeom sg;
};

// The 8 sequence ids [8*lane, 8*lane+8) of a stage's id tile.
__device__ __forceinline__ void lds_ids(const unsigned char* ids, int lane, int (&v)[8]) {
  const int4* p = reinterpret_cast<const int4*>(ids) + 2 * lane;
  const int4 a = p[0], b = p[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Halo ids of a lane (positions 8*lane-H .. 8*lane-1): from lane-1, or for
// lane 0 from the previous tile (carry, updated to this tile's last ids).
template <int H>
__device__ __forceinline__ void ids_halo(const int (&sid)[8], int (&carry)[H], int (&hs)[H], int lane) {
#pragma unroll
  for (int j = 0; j < H; ++j) {
    const int up = __shfl_up_sync(kFull, sid[8 - H + j], 1);
    const int nc = __shfl_sync(kFull, sid[8 - H + j], 31);
    hs[j] = lane == 0 ? carry[j] : up;
    carry[j] = nc;
  }
}

// True when the whole warp's 8 positions and their halos carry one
// non-negative id: no sequence boundary, no padding -- the ungated math
// applies.
template <int H>
__device__ __forceinline__ bool ids_uniform(const int (&sid)[8], const int (&hs)[H]) {
  const int s0 = sid[0];
  bool u = s0 >= 0;
#pragma unroll
  for (int i = 1; i < 8; ++i) u = u && sid[i] == s0;
#pragma unroll
  for (int j = 0; j < H; ++j) u = u && hs[j] == s0;
  return __all_sync(kFull, u);
}

// seq_idx at position q (kNoSeq outside 0 .. L-1).
__device__ __forceinline__ int seq_at(const int* seq, i64 ss_l, i64 q, i64 L) {
  return (q >= 0 && q < L) ? seq[q * ss_l] : kNoSeq;
}

// The 8 positions [8*lane, 8*lane+8) of tile row r, converted to float.
template <typename T>
__device__ __forceinline__ void lds8(const unsigned char* tile, int r, int lane, float (&v)[8]) {
  const T* p = reinterpret_cast<const T*>(tile) + r * kTL + lane * 8;
  if constexpr (sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Pair<T>::unpack(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Stores 8 consecutive elements (16-byte aligned for 16-bit types).
template <typename T>
__device__ __forceinline__ void stg8(T* p, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    u.x = Pair<T>::pack(f2(v[0], v[1]));
    u.y = Pair<T>::pack(f2(v[2], v[3]));
    u.z = Pair<T>::pack(f2(v[4], v[5]));
    u.w = Pair<T>::pack(f2(v[6], v[7]));
    *reinterpret_cast<uint4*>(p) = u;
  } else {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__device__ __forceinline__ float2 shfl_up2(float2 v, int d) {
  return f2(__shfl_up_sync(kFull, v.x, d), __shfl_up_sync(kFull, v.y, d));
}
__device__ __forceinline__ float2 shfl_down2(float2 v, int d) {
  return f2(__shfl_down_sync(kFull, v.x, d), __shfl_down_sync(kFull, v.y, d));
}
__device__ __forceinline__ float2 shfl2(float2 v, int src) {
  return f2(__shfl_sync(kFull, v.x, src), __shfl_sync(kFull, v.y, src));
}

// xc (x preceded by initial_states or zeros) at position q of rows (ra, rb).
template <typename T>
__device__ __forceinline__ float2 xc_pair(const T* x, i64 xs_c, i64 xs_l, const T* init, i64 is_c, i64 is_l,
                                          int H, i64 q, bool va, bool vb) {
  float2 r = f2(0.f, 0.f);
  if (q >= 0) {
    if (va) r.x = Cvt<T>::f(x[q * xs_l]);
    if (vb) r.y = Cvt<T>::f(x[xs_c + q * xs_l]);
  } else if (init != nullptr) {
    if (va) r.x = Cvt<T>::f(init[(q + H) * is_l]);
    if (vb) r.y = Cvt<T>::f(init[is_c + (q + H) * is_l]);
  }
  return r;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

template <typename T, int W, bool HAS_SEQ, bool SILU>
__global__ void __launch_bounds__(kThreadsSeq, (sizeof(T) == 2 && !HAS_SEQ && W <= 7) ? CC1D_SEQ_FWD_FAST_MIN_BLOCKS : CC1D_SEQ_FWD_MIN_BLOCKS) fwd_seq_tma_kernel(const __grid_constant__ SeqFwdParams p) {
  constexpr int H = W - 1;
  constexpr unsigned TB = seq_tile_bytes<T>();
  constexpr unsigned SB = TB + (HAS_SEQ ? kIdsBytes : 0u);
  constexpr int NS = seq_fwd_stages<T>();
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  const FwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 item = blockIdx.x;
  const i64 seg = item % a.nseg;
  const i64 rest = item / a.nseg;
  const i64 grp = rest % p.groups;
  const i64 b = rest / p.groups;
  const i64 c0 = grp * kRows;
  const i64 t0 = seg * a.seg_len;
  const i64 t1 = min(a.L, t0 + a.seg_len);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // inputs of this launch may come from the previous kernel
  griddep_launch_dependents();

  if (warp == kSW) {
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      if (HAS_SEQ) prefetch_tensormap(&p.map_s);
      unsigned k = 0;
      for (i64 t = t0; t < t1; t += kTL, ++k) {
        const unsigned s = k % NS, use = k / NS;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) break;  // consumers stopped
        mbar_arrive_expect_tx(&full[s], SB);
        tma_load_3d(smem + s * SB, &p.map_x, &full[s], (int)t, (int)c0, (int)b);
        if (HAS_SEQ) tma_load_3d(smem + s * SB + TB, &p.map_s, &full[s], (int)t, 0, (int)b);
      }
      mbar_drain(full, k, NS);
    }
    return;
  }

  const i64 ra = c0 + 2 * warp;  // rows (channels) of this warp: ra, ra + 1
  const bool va = ra < a.D, vb = ra + 1 < a.D;
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  float2 wp[W];
#pragma unroll
  for (int k = 0; k < W; ++k)
    wp[k] = f2(va ? Cvt<T>::f(wt[ra * a.ws_c + k * a.ws_k]) : 0.f, vb ? Cvt<T>::f(wt[(ra + 1) * a.ws_c + k * a.ws_k]) : 0.f);
  const float2 bp = f2((bias && va) ? Cvt<T>::f(bias[ra * a.bs]) : 0.f, (bias && vb) ? Cvt<T>::f(bias[(ra + 1) * a.bs]) : 0.f);
  const T* __restrict__ xr = static_cast<const T*>(a.x) + b * a.xs_b + ra * a.xs_c;
  const T* __restrict__ ir = a.init ? static_cast<const T*>(a.init) + b * a.is_b + ra * a.is_c : nullptr;
  T* __restrict__ oa = static_cast<T*>(a.out) + b * a.os_b + ra * a.os_c;

  // Halo of lane 0 in the first tile: xc at t0-H .. t0-1 (and its ids).
  float2 carry[H];
#pragma unroll
  for (int j = 0; j < H; ++j) carry[j] = xc_pair(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, t0 - H + j, va, vb);
  const int* __restrict__ seq = HAS_SEQ ? a.seq + b * a.ss_b : nullptr;
  int scarry[H];
#pragma unroll
  for (int j = 0; j < H; ++j) scarry[j] = HAS_SEQ ? seq_at(seq, a.ss_l, t0 - H + j, a.L) : 0;

  unsigned k = 0;
  for (i64 t = t0; t < t1; t += kTL, ++k) {
    const unsigned s = k % NS, use = k / NS;
    if (!mbar_wait(&full[s], use & 1)) return;
    float xa[8], xb[8];
    lds8<T>(smem + s * SB, 2 * warp, lane, xa);
    lds8<T>(smem + s * SB, 2 * warp + 1, lane, xb);
    int sid[8];
    if (HAS_SEQ) lds_ids(smem + s * SB + TB, lane, sid);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float2 xp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xp[i] = f2(xa[i], xb[i]);
    float2 h[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const float2 up = shfl_up2(xp[8 - H + j], 1);
      const float2 nc = shfl2(xp[8 - H + j], 31);
      h[j] = lane == 0 ? carry[j] : up;
      carry[j] = nc;
    }
    int hs[H];
    bool gated = false;
    if (HAS_SEQ) {
      ids_halo<H>(sid, scarry, hs, lane);
      gated = !ids_uniform<H>(sid, hs);
    }
    float oa8[8], ob8[8];
    if (!gated) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 acc = bp;
#pragma unroll
        for (int kk = 0; kk < W; ++kk) {
          const int q = i - H + kk;
          acc = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], acc);
        }
        if (SILU) acc = silu2(acc);
        oa8[i] = acc.x;
        ob8[i] = acc.y;
      }
    } else {
      // A tap counts only when its position carries the output's sequence
      // id; padding positions (id < 0) output 0.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int si = sid[i];
        float2 acc = bp;
#pragma unroll
        for (int kk = 0; kk < W; ++kk) {
          const int q = i - H + kk;
          const int sq = q >= 0 ? sid[q >= 0 ? q : 0] : hs[q >= 0 ? 0 : q + H];
          if (sq == si) acc = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], acc);
        }
        if (SILU) acc = silu2(acc);
        if (si < 0) acc = f2(0.f, 0.f);
        oa8[i] = acc.x;
        ob8[i] = acc.y;
      }
    }
    const i64 pos = t + 8 * lane;
    if (pos < t1) {
      if (va) stg8<T>(oa + pos, oa8);
      if (vb) stg8<T>(oa + a.os_c + pos, ob8);
    }
  }
  if (a.fin != nullptr && t1 == a.L && lane < H) {
    T* f = static_cast<T*>(a.fin) + b * a.fs_b + ra * a.fs_c + lane * a.fs_l;
    const i64 q = a.L - H + lane;
    const float2 v = xc_pair(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, q, va, vb);
    if (va) f[0] = Cvt<T>::to(v.x);
    if (vb) f[a.fs_c] = Cvt<T>::to(v.y);
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// dx of the 8 positions of a lane from dpre of those positions (d) and of the
// H positions after them (rh), plus dfinal where final_states read them.
template <typename T, int W>
__device__ __forceinline__ void emit_dx(const float2 (&d)[8], const float2 (&rh)[W - 1], const float2 (&wp)[W],
                                        i64 pos, bool store, const BwdArgs& a, T* dxa, const T* fa, bool va, bool vb) {
  constexpr int H = W - 1;
  float ea[8], eb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m <= H; ++m) {
      const int q = i + m;
      acc = fma2(wp[H - m], q < 8 ? d[q < 8 ? q : 0] : rh[q < 8 ? 0 : q - 8], acc);
    }
    ea[i] = acc.x;
    eb[i] = acc.y;
  }
  // dfinal_states reach only the last W-1 positions of the sequence.
  if (fa != nullptr && pos + 8 + H > a.L) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const i64 qf = pos + i + H - a.L;
      if (qf >= 0 && pos + i < a.L) {
        if (va) ea[i] += Cvt<T>::f(fa[qf * a.fs_l]);
        if (vb) eb[i] += Cvt<T>::f(fa[a.fs_c + qf * a.fs_l]);
      }
    }
  }
  if (store) {
    if (va) stg8<T>(dxa + pos, ea);
    if (vb) stg8<T>(dxa + a.dxs_c + pos, eb);
  }
}

// emit_dx with seq_idx: dx at position q sums the taps of the outputs q+m
// that carry q's sequence id -- bit m-1 of the mask of q+m (dpre is already 0
// at padding).  m: this lane's masks; rm: the masks of the next lane's first
// positions (words 0 .. 3).
template <typename T, int W>
__device__ __forceinline__ void emit_dx_mask(const float2 (&d)[8], const float2 (&rh)[W - 1], const uint32_t (&m)[4],
                                             const uint32_t (&rm)[4], const float2 (&wp)[W], i64 pos, bool store,
                                             T* dxa, i64 dxs_c, bool va, bool vb) {
  constexpr int H = W - 1;
  float ea[8], eb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k <= H; ++k) {
      const int q = i + k;
      const uint32_t mq = q < 8 ? mask_at(m, q < 8 ? q : 0) : mask_at(rm, q < 8 ? 0 : q - 8);
      if (k == 0 || ((mq >> (k - 1)) & 1u)) acc = fma2(wp[H - k], q < 8 ? d[q < 8 ? q : 0] : rh[q < 8 ? 0 : q - 8], acc);
    }
    ea[i] = acc.x;
    eb[i] = acc.y;
  }
  if (store) {
    if (va) stg8<T>(dxa + pos, ea);
    if (vb) stg8<T>(dxa + dxs_c + pos, eb);
  }
}

// The backward's tiles overlap by one lane: a tile holds 256 positions
// [t, t + 256) but the walk advances kBwdStep = 248, so lanes 0..30 own
// [t, t + 248) and lane 31 only recomputes dpre of [t + 248, t + 256) -- the
// right halo of lane 30's dx, owned by the next tile.  Every tile's dx is
// therefore emitted within the tile (no dpre carried to the next one), and
// a segment's last tile already holds the dpre just past the segment, where
// lane 31 (or the lanes past the segment end) compute it from the tile like
// any other position.  The overlap costs 1/32 of the arithmetic and an
// 8-position L2 re-read per tile; it frees the registers of a tile of
// delayed dpre and the scalar loads of the segment's tail.
template <typename T, int W, bool HAS_SEQ, bool SILU>
__global__ void __launch_bounds__(kThreadsSeq, W > 5 ? 1 : (HAS_SEQ ? CC1D_SEQ_BWD_IDS_MIN_BLOCKS : CC1D_SEQ_BWD_MIN_BLOCKS)) bwd_seq_tma_kernel(const __grid_constant__ SeqBwdParams p) {
  constexpr int H = W - 1;
  constexpr unsigned TB = seq_tile_bytes<T>();
  constexpr unsigned SB = 2 * TB + (HAS_SEQ ? kMaskBytes : 0u);
  constexpr int NS = seq_bwd_stages<T>();
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  const BwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 item = blockIdx.x;
  const i64 seg = item % a.nseg;
  const i64 rest = item / a.nseg;
  const i64 grp = rest % p.groups;
  const i64 b = rest / p.groups;
  const i64 c0 = grp * kRows;
  const i64 t0 = seg * a.seg_len;
  const i64 t1 = min(a.L, t0 + a.seg_len);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // inputs of this launch may come from the previous kernel
  griddep_launch_dependents();

  if (warp == kSW) {
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      prefetch_tensormap(&p.map_g);
      if (HAS_SEQ) prefetch_tensormap(&p.map_s);
      unsigned k = 0;
      for (i64 t = t0; t < t1; t += kBwdStep, ++k) {
        const unsigned s = k % NS, use = k / NS;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) break;  // consumers stopped
        mbar_arrive_expect_tx(&full[s], SB);
        tma_load_3d(smem + s * SB, &p.map_x, &full[s], (int)t, (int)c0, (int)b);
        tma_load_3d(smem + s * SB + TB, &p.map_g, &full[s], (int)t, (int)c0, (int)b);
        if (HAS_SEQ) tma_load_3d(smem + s * SB + 2 * TB, &p.map_s, &full[s], (int)t, 0, (int)b);
      }
      mbar_drain(full, k, NS);
    }
    return;
  }

  const i64 ra = c0 + 2 * warp;
  const bool va = ra < a.D, vb = ra + 1 < a.D;
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  float2 wp[W];
#pragma unroll
  for (int k = 0; k < W; ++k)
    wp[k] = f2(va ? Cvt<T>::f(wt[ra * a.ws_c + k * a.ws_k]) : 0.f, vb ? Cvt<T>::f(wt[(ra + 1) * a.ws_c + k * a.ws_k]) : 0.f);
  const float2 bp = f2((bias && va) ? Cvt<T>::f(bias[ra * a.bs]) : 0.f, (bias && vb) ? Cvt<T>::f(bias[(ra + 1) * a.bs]) : 0.f);
  const T* __restrict__ xr = static_cast<const T*>(a.x) + b * a.xs_b + ra * a.xs_c;
  const T* __restrict__ ir = a.init ? static_cast<const T*>(a.init) + b * a.is_b + ra * a.is_c : nullptr;
  const T* __restrict__ fa = a.dfin ? static_cast<const T*>(a.dfin) + b * a.fs_b + ra * a.fs_c : nullptr;
  T* __restrict__ dxa = static_cast<T*>(a.dx) + b * a.dxs_b + ra * a.dxs_c;

  // Halo of lane 0 in the first tile: xc at t0-H .. t0-1.
  float2 carry[H];
#pragma unroll
  for (int j = 0; j < H; ++j) carry[j] = xc_pair(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, t0 - H + j, va, vb);

  float2 dw[W];
#pragma unroll
  for (int k = 0; k < W; ++k) dw[k] = f2(0.f, 0.f);
  float2 db = f2(0.f, 0.f);

  unsigned k = 0;
  for (i64 t = t0; t < t1; t += kBwdStep, ++k) {
    const unsigned s = k % NS, use = k / NS;
    if (!mbar_wait(&full[s], use & 1)) return;
    float xa[8], xb[8], ga[8], gb[8];
    lds8<T>(smem + s * SB, 2 * warp, lane, xa);
    lds8<T>(smem + s * SB, 2 * warp + 1, lane, xb);
    lds8<T>(smem + s * SB + TB, 2 * warp, lane, ga);
    lds8<T>(smem + s * SB + TB, 2 * warp + 1, lane, gb);
    uint32_t mk[4];
    if (HAS_SEQ) lds_masks(smem + s * SB + 2 * TB, lane, mk);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    float2 xp[8], d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xp[i] = f2(xa[i], xb[i]);
    // Left halo from lane - 1; lane 0 takes the previous tile's lane 30.
    float2 h[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const float2 up = shfl_up2(xp[8 - H + j], 1);
      const float2 nc = shfl2(xp[8 - H + j], 31 - 1);
      h[j] = lane == 0 ? carry[j] : up;
      carry[j] = nc;
    }
    // Gated when any mask of the tile is not full.  A full tile also makes
    // every dx tap of lanes 0..30 count (their right halos lie in the tile).
    bool gated = false;
    if (HAS_SEQ) {
      constexpr uint32_t kFull2 = mask_full<H>() * 0x10001u;
      gated = !__all_sync(kFull, (mk[0] & mk[1] & mk[2] & mk[3]) == kFull2);
    }
    const i64 pos = t + 8 * lane;
    const bool own = lane < 31 && pos < t1;  // positions whose dx, dweight and dbias this tile produces
    if (!gated) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 pre = bp;
#pragma unroll
        for (int kk = 0; kk < W; ++kk) {
          const int q = i - H + kk;
          pre = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], pre);
        }
        const float2 g = f2(ga[i], gb[i]);
        d[i] = SILU ? mul2(g, silu_grad2(pre)) : g;
        if (own) {
          db = add2(db, d[i]);
#pragma unroll
          for (int kk = 0; kk < W; ++kk) {
            const int q = i - H + kk;
            dw[kk] = fma2(d[i], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], dw[kk]);
          }
        }
      }
    } else {
      // Tap kk of output i counts when mask bit H-1-kk of i is set (the
      // position H-kk before it carries its id); dpre is 0 at padding.
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t mi = mask_at(mk, i);
        float2 pre = bp;
#pragma unroll
        for (int kk = 0; kk < W; ++kk) {
          const int q = i - H + kk;
          if (kk == H || ((mi >> (H - 1 - kk)) & 1u))
            pre = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], pre);
        }
        const float2 g = f2(ga[i], gb[i]);
        d[i] = SILU ? mul2(g, silu_grad2(pre)) : g;
        if (!(mi & kMaskValid)) d[i] = f2(0.f, 0.f);
        if (own) {
          db = add2(db, d[i]);
#pragma unroll
          for (int kk = 0; kk < W; ++kk) {
            const int q = i - H + kk;
            if (kk == H || ((mi >> (H - 1 - kk)) & 1u))
              dw[kk] = fma2(d[i], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], dw[kk]);
          }
        }
      }
    }
    // dx of this tile: the right halo of lane l is lane l + 1's first dpre
    // (lane 30 reads the overlap lane; lane 31 stores nothing).
    float2 rh[H];
#pragma unroll
    for (int j = 0; j < H; ++j) rh[j] = shfl_down2(d[j], 1);
    if (gated) {
      uint32_t rm[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) rm[w] = 2 * w < H ? __shfl_down_sync(kFull, mk[w], 1) : 0u;
      emit_dx_mask<T, W>(d, rh, mk, rm, wp, pos, own, dxa, a.dxs_c, va, vb);
    } else {
      emit_dx<T, W>(d, rh, wp, pos, own, a, dxa, fa, va, vb);
    }
    // dinitial_states: dpre of positions 0 .. H-1 live in lane 0 of tile 0.
    if (t == 0 && lane == 0 && a.dinit != nullptr) {
      T* di = static_cast<T*>(a.dinit) + b * a.dis_b + ra * a.dis_c;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float2 acc = f2(0.f, 0.f);
#pragma unroll
        for (int kk = 0; kk <= i; ++kk) acc = fma2(wp[kk], d[i - kk], acc);
        if (fa != nullptr && i - a.L >= 0) {
          if (va) acc.x += Cvt<T>::f(fa[(i - a.L) * a.fs_l]);
          if (vb) acc.y += Cvt<T>::f(fa[a.fs_c + (i - a.L) * a.fs_l]);
        }
        if (va) di[i * a.dis_l] = Cvt<T>::to(acc.x);
        if (vb) di[a.dis_c + i * a.dis_l] = Cvt<T>::to(acc.y);
      }
    }
  }
  // Warp sums of the dweight / dbias partials; lane 0 writes this item's slot.
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int kk = 0; kk < W; ++kk) dw[kk] = add2(dw[kk], shfl_down2(dw[kk], off));
    db = add2(db, shfl_down2(db, off));
  }
  if (lane == 0) {
    float* pp = a.partials + ((b * a.nseg + seg) * a.D + ra) * (W + 1);
    if (va) {
#pragma unroll
      for (int kk = 0; kk < W; ++kk) pp[kk] = dw[kk].x;
      pp[W] = db.x;
    }
    if (vb) {
#pragma unroll
      for (int kk = 0; kk < W; ++kk) pp[W + 1 + kk] = dw[kk].y;
      pp[W + 1 + W] = db.y;
    }
  }
}

// ---------------------------------------------------------------------------
// Rows whose pitch is not a multiple of 16 bytes ("shifted" rows)
// ---------------------------------------------------------------------------
// TMA cannot describe such rows with a 3-D map (strides must be multiples of
// 16 bytes).  The tensor is then viewed as a 2-D array of view rows of `in`
// elements (the largest power of two of at most 128 bytes that divides the
// tensor's extent), and the tiles of a channel row are laid on the tensor's
// own 16-byte grid instead of on the row's start: with off = the offset of
// the row's position 0 in its 16-byte unit (0 .. E-1, E = 16 / sizeof(T)),
// the row's tiles begin at positions seg_start - off + 256 j.  Every lane's
// 8 elements are then one aligned vector, in shared memory and in global
// memory, and nothing is realigned.  A tile is one box of kTL / in + 1 view
// rows starting at the view row that holds the tile's first element, which
// sits o2 (a multiple of E) elements into the box.
//
// The first tile of a row holds, at positions -off .. -1, the end of the
// previous row: lane 0 overwrites those elements in shared memory with xc
// there (initial states or zeros); outputs there are not stored and dpre
// there is 0.  Past L a tile holds the next row: stores are masked and dpre
// is 0.  Segment bounds move with the row (seg_start - off), so segments
// still partition the row; the two rows of a warp, whose offsets differ,
// share every lane's frame index and keep their own positions.

// Largest view row, in bytes.  A box is kTL * sizeof(T) + (view row) bytes.
constexpr int kShMaxRowBytes = 128;

template <typename T>
constexpr int unit_elems() {
  return 16 / (int)sizeof(T);
}
// smem bytes of one shifted row tile: the largest box.
template <typename T>
constexpr unsigned sh_row_bytes() {
  return ((unsigned)(kTL * sizeof(T) + kShMaxRowBytes) + 127u) / 128u * 128u;  // 640 or 1152
}

// xc (x preceded by initial_states or zeros) of one row at position q.
template <typename T>
__device__ __forceinline__ float xc_one(const T* x, i64 xs_l, const T* init, i64 is_l, int H, int q) {
  if (q >= 0) return Cvt<T>::f(x[q * xs_l]);
  if (init != nullptr && q >= -H) return Cvt<T>::f(init[(q + H) * is_l]);
  return 0.f;
}

// xc of rows (ra, ra + 1) at their own positions qa, qb.
template <typename T>
__device__ __forceinline__ float2 xc_rows(const T* x, i64 xs_c, i64 xs_l, const T* init, i64 is_c, i64 is_l, int H,
                                          int qa, int qb, bool va, bool vb) {
  return f2(va ? xc_one(x, xs_l, init, is_l, H, qa) : 0.f,
            vb ? xc_one(x + xs_c, xs_l, init != nullptr ? init + is_c : nullptr, is_l, H, qb) : 0.f);
}

// The 8 elements [8*lane, 8*lane+8) of a row tile that starts at `row`
// (16-byte aligned), as floats.
template <typename T>
__device__ __forceinline__ void lds8_row(const unsigned char* row, int lane, float (&v)[8]) {
  const T* p = reinterpret_cast<const T*>(row) + lane * 8;
  if constexpr (sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Pair<T>::unpack(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Stores a lane's 8 values at row positions [q, q + 8) (q + row start on the
// 16-byte grid): one vector when all lie in [0, L), else the ones that do.
template <typename T>
__device__ __forceinline__ void stg8_rowpos(T* row, int q, int L, const float (&v)[8]) {
  if (q >= 0 && q + 8 <= L) {
    stg8<T>(row + q, v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (q + i >= 0 && q + i < L) row[q + i] = Cvt<T>::to(v[i]);
  }
}

// First tile of a row: its positions -off .. -1 hold the previous row's
// elements; lane 0 overwrites them in shared memory with xc there (initial
// states or zeros).  The caller orders these writes before the stage's next
// TMA with a proxy fence.
template <typename T>
__device__ __forceinline__ void fix_row_head(unsigned char* row, int off, const T* init, i64 is_l, int H) {
  T* e = reinterpret_cast<T*>(row);
  for (int i = 0; i < off; ++i) {
    const int q = i - off;
    e[i] = (init != nullptr && q >= -H) ? init[(q + H) * is_l] : Cvt<T>::to(0.f);
  }
}

// Producer: one box per channel row of the group, at the view row holding
// the row's first tile element (rows past D read whatever lies there or the
// fill value; nothing is stored for them).
__device__ __forceinline__ void shift_load_rows(unsigned char* dst, unsigned row_bytes, const CUtensorMap* map,
                                                uint64_t* bar, i64 rbase, i64 s_c, int t, int E, int in_log2) {
#pragma unroll 1
  for (int r = 0; r < kRows; ++r) {
    const i64 e0 = ((rbase + r * s_c) & ~(i64)(E - 1)) + t;
    tma_load_3d(dst + r * row_bytes, map, bar, 0, (int)(e0 >> in_log2), 0);
  }
}

template <typename T, int W, bool SILU>
__global__ void __launch_bounds__(kThreadsSeq, CC1D_SEQ_FWD_SH_MIN_BLOCKS) fwd_shift_tma_kernel(const __grid_constant__ SeqFwdParams p) {
  constexpr int H = W - 1;
  constexpr int E = unit_elems<T>();
  constexpr unsigned RB = sh_row_bytes<T>();
  constexpr unsigned SB = kRows * RB;
  constexpr int NS = seq_fwd_stages<T>();
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  const FwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 item = blockIdx.x;
  const i64 seg = item % a.nseg;
  const i64 rest = item / a.nseg;
  const i64 grp = rest % p.groups;
  const i64 b = rest / p.groups;
  const i64 c0 = grp * kRows;
  // Positions fit 32 bits (L < 2^31 - 2^12).
  const int L = (int)a.L, seg_len = (int)a.seg_len;
  const int t0 = (int)seg * seg_len;
  const bool last_seg = seg == a.nseg - 1;
  const int ntiles = last_seg ? p.sg.tiles_last : p.sg.tiles_full;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // inputs of this launch may come from the previous kernel
  griddep_launch_dependents();

  if (warp == kSW) {
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      const i64 rbase = b * a.xs_b + c0 * a.xs_c;
      int k = 0;
      for (; k < ntiles; ++k) {
        const unsigned s = k % NS, use = k / NS;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) break;  // consumers stopped
        mbar_arrive_expect_tx(&full[s], p.sg.tx);
        shift_load_rows(smem + s * SB, RB, &p.map_x, &full[s], rbase, a.xs_c, t0 + k * kTL, E, p.sg.in_log2);
      }
      mbar_drain(full, (unsigned)k, NS);
    }
    return;
  }

  const i64 ra = c0 + 2 * warp;  // rows (channels) of this warp: ra, ra + 1
  const bool va = ra < a.D, vb = ra + 1 < a.D;
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  float2 wp[W];
#pragma unroll
  for (int k = 0; k < W; ++k)
    wp[k] = f2(va ? Cvt<T>::f(wt[ra * a.ws_c + k * a.ws_k]) : 0.f, vb ? Cvt<T>::f(wt[(ra + 1) * a.ws_c + k * a.ws_k]) : 0.f);
  const float2 bp = f2((bias && va) ? Cvt<T>::f(bias[ra * a.bs]) : 0.f, (bias && vb) ? Cvt<T>::f(bias[(ra + 1) * a.bs]) : 0.f);
  const i64 Ra = b * a.xs_b + ra * a.xs_c, Rb = Ra + a.xs_c;  // element index of each row's position 0
  const int off_a = (int)(Ra & (E - 1)), off_b = (int)(Rb & (E - 1));
  const unsigned o2a = (unsigned)((Ra & (p.sg.in - 1)) - off_a) * sizeof(T);
  const unsigned o2b = (unsigned)((Rb & (p.sg.in - 1)) - off_b) * sizeof(T);
  const T* __restrict__ xr = static_cast<const T*>(a.x) + Ra;
  const T* __restrict__ ir = a.init ? static_cast<const T*>(a.init) + b * a.is_b + ra * a.is_c : nullptr;
  T* __restrict__ oa = static_cast<T*>(a.out) + Ra;  // out has x's strides
  T* __restrict__ ob = oa + a.xs_c;
  // Row positions of this lane's element 0 in the segment's first tile.
  const int qa0 = t0 - off_a + 8 * lane, qb0 = t0 - off_b + 8 * lane;

  // Halo of lane 0 in the first tile: xc before each row's first tile.
  float2 carry[H];
#pragma unroll
  for (int j = 0; j < H; ++j)
    carry[j] = xc_rows(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, t0 - off_a - H + j, t0 - off_b - H + j, va, vb);

  for (int k = 0; k < ntiles; ++k) {
    const unsigned s = k % NS, use = k / NS;
    if (!mbar_wait(&full[s], use & 1)) return;
    unsigned char* rowa = smem + s * SB + (2 * warp) * RB + o2a;
    unsigned char* rowb = smem + s * SB + (2 * warp + 1) * RB + o2b;
    if (t0 == 0 && k == 0) {
      if (lane == 0) {
        if (va) fix_row_head<T>(rowa, off_a, ir, a.is_l, H);
        if (vb) fix_row_head<T>(rowb, off_b, ir != nullptr ? ir + a.is_c : nullptr, a.is_l, H);
        fence_proxy_async_smem();
      }
      __syncwarp();
    }
    float xa[8], xb[8];
    lds8_row<T>(rowa, lane, xa);
    lds8_row<T>(rowb, lane, xb);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const int qa = qa0 + k * kTL, qb = qb0 + k * kTL;
    float2 xp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xp[i] = f2(xa[i], xb[i]);
    float2 h[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const float2 up = shfl_up2(xp[8 - H + j], 1);
      const float2 nc = shfl2(xp[8 - H + j], 31);
      h[j] = lane == 0 ? carry[j] : up;
      carry[j] = nc;
    }
    float oa8[8], ob8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 acc = bp;
#pragma unroll
      for (int kk = 0; kk < W; ++kk) {
        const int q = i - H + kk;
        acc = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], acc);
      }
      if (SILU) acc = silu2(acc);
      oa8[i] = acc.x;
      ob8[i] = acc.y;
    }
    if (va) stg8_rowpos<T>(oa, qa, L, oa8);
    if (vb) stg8_rowpos<T>(ob, qb, L, ob8);
  }
  if (a.fin != nullptr && last_seg && lane < H) {
    T* f = static_cast<T*>(a.fin) + b * a.fs_b + ra * a.fs_c + lane * a.fs_l;
    const i64 q = a.L - H + lane;
    const float2 v = xc_pair(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, q, va, vb);
    if (va) f[0] = Cvt<T>::to(v.x);
    if (vb) f[a.fs_c] = Cvt<T>::to(v.y);
  }
}

// dpre of rows (ra, ra + 1) at their own positions qa, qb (0 at or past L).
template <typename T, int W, bool SILU>
__device__ __forceinline__ float2 dpre_rows(const T* xr, const T* gr, const T* ir, const BwdArgs& a,
                                            const float2 (&wp)[W], float2 bp, int qa, int qb, bool va, bool vb) {
  constexpr int H = W - 1;
  const bool ia = va && qa < (int)a.L, ib = vb && qb < (int)a.L;  // nothing is read past the row
  float2 pre = bp;
#pragma unroll
  for (int kk = 0; kk < W; ++kk)
    pre = fma2(wp[kk], xc_rows(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, qa - H + kk, qb - H + kk, ia, ib), pre);
  const float2 g = f2(ia ? Cvt<T>::f(gr[qa]) : 0.f, ib ? Cvt<T>::f(gr[a.xs_c + qb]) : 0.f);
  return SILU ? mul2(g, silu_grad2(pre)) : g;
}

// dx of a lane's 8 positions (rows at qa, qb) from dpre of those positions
// (d) and of the H positions after them (rh), plus dfinal where final_states
// read them; stored within [0, L).
template <typename T, int W>
__device__ __forceinline__ void emit_dx_shift(const float2 (&d)[8], const float2 (&rh)[W - 1], const float2 (&wp)[W],
                                              int qa, int qb, int L, const BwdArgs& a, T* dxa, const T* fa, bool va,
                                              bool vb) {
  constexpr int H = W - 1;
  float ea[8], eb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m <= H; ++m) {
      const int q = i + m;
      acc = fma2(wp[H - m], q < 8 ? d[q < 8 ? q : 0] : rh[q < 8 ? 0 : q - 8], acc);
    }
    ea[i] = acc.x;
    eb[i] = acc.y;
  }
  if (fa != nullptr && (qa + 8 + H > L || qb + 8 + H > L)) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int fqa = qa + i + H - L, fqb = qb + i + H - L;
      if (va && fqa >= 0 && qa + i < L) ea[i] += Cvt<T>::f(fa[fqa * a.fs_l]);
      if (vb && fqb >= 0 && qb + i < L) eb[i] += Cvt<T>::f(fa[a.fs_c + fqb * a.fs_l]);
    }
  }
  if (va) stg8_rowpos<T>(dxa, qa, L, ea);
  if (vb) stg8_rowpos<T>(dxa + a.xs_c, qb, L, eb);
}

// Like bwd_seq_tma_kernel, the tiles overlap by one lane (they advance
// kBwdStep = 248 positions): lanes 0..30 own their positions, lane 31
// recomputes the dpre lane 30's dx needs, and each tile's dx is emitted in
// the tile.  A tile's first element then sits at a different offset of its
// box from tile to tile (248 is not a multiple of the view row).
template <typename T, int W, bool SILU>
__global__ void __launch_bounds__(kThreadsSeq, W > 5 ? 1 : CC1D_SEQ_BWD_SH_MIN_BLOCKS) bwd_shift_tma_kernel(const __grid_constant__ SeqBwdParams p) {
  constexpr int H = W - 1;
  constexpr int E = unit_elems<T>();
  constexpr unsigned RB = sh_row_bytes<T>();
  constexpr unsigned TB = kRows * RB;
  constexpr unsigned SB = 2 * TB;
  constexpr int NS = seq_bwd_stages<T>();
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + NS;
  const BwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 item = blockIdx.x;
  const i64 seg = item % a.nseg;
  const i64 rest = item / a.nseg;
  const i64 grp = rest % p.groups;
  const i64 b = rest / p.groups;
  const i64 c0 = grp * kRows;
  const int L = (int)a.L, seg_len = (int)a.seg_len;
  const int t0 = (int)seg * seg_len;
  const bool last_seg = seg == a.nseg - 1;
  const int ntiles = last_seg ? p.sg.tiles_last : p.sg.tiles_full;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();

  if (warp == kSW) {
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      prefetch_tensormap(&p.map_g);
      const i64 rbase = b * a.xs_b + c0 * a.xs_c;  // dout and dx have x's strides
      int k = 0;
      for (; k < ntiles; ++k) {
        const unsigned s = k % NS, use = k / NS;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) break;  // consumers stopped
        mbar_arrive_expect_tx(&full[s], 2 * p.sg.tx);
        const int t = t0 + k * kBwdStep;
        shift_load_rows(smem + s * SB, RB, &p.map_x, &full[s], rbase, a.xs_c, t, E, p.sg.in_log2);
        shift_load_rows(smem + s * SB + TB, RB, &p.map_g, &full[s], rbase, a.xs_c, t, E, p.sg.in_log2);
      }
      mbar_drain(full, (unsigned)k, NS);
    }
    return;
  }

  const i64 ra = c0 + 2 * warp;
  const bool va = ra < a.D, vb = ra + 1 < a.D;
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  float2 wp[W];
#pragma unroll
  for (int k = 0; k < W; ++k)
    wp[k] = f2(va ? Cvt<T>::f(wt[ra * a.ws_c + k * a.ws_k]) : 0.f, vb ? Cvt<T>::f(wt[(ra + 1) * a.ws_c + k * a.ws_k]) : 0.f);
  const float2 bp = f2((bias && va) ? Cvt<T>::f(bias[ra * a.bs]) : 0.f, (bias && vb) ? Cvt<T>::f(bias[(ra + 1) * a.bs]) : 0.f);
  const i64 Ra = b * a.xs_b + ra * a.xs_c, Rb = Ra + a.xs_c;
  const int off_a = (int)(Ra & (E - 1)), off_b = (int)(Rb & (E - 1));
  // Low bits of each row's aligned start: with the tile's start they give the
  // tile's first element within its box.
  const unsigned ba = (unsigned)(Ra - off_a), bb = (unsigned)(Rb - off_b);
  const unsigned inm = (unsigned)p.sg.in - 1u;
  const T* __restrict__ xr = static_cast<const T*>(a.x) + Ra;
  const T* __restrict__ gr = static_cast<const T*>(a.dout) + Ra;
  const T* __restrict__ ir = a.init ? static_cast<const T*>(a.init) + b * a.is_b + ra * a.is_c : nullptr;
  T* __restrict__ dxa = static_cast<T*>(a.dx) + Ra;
  const T* __restrict__ fa = a.dfin ? static_cast<const T*>(a.dfin) + b * a.fs_b + ra * a.fs_c : nullptr;
  const int qa0 = t0 - off_a + 8 * lane, qb0 = t0 - off_b + 8 * lane;

  float2 carry[H];
#pragma unroll
  for (int j = 0; j < H; ++j)
    carry[j] = xc_rows(xr, a.xs_c, a.xs_l, ir, a.is_c, a.is_l, H, t0 - off_a - H + j, t0 - off_b - H + j, va, vb);
  // dinitial_states from dpre of positions 0 .. H-1, read directly.
  if (t0 == 0 && a.dinit != nullptr) {
    float2 dq[H];
#pragma unroll
    for (int i = 0; i < H; ++i) dq[i] = dpre_rows<T, W, SILU>(xr, gr, ir, a, wp, bp, i, i, va, vb);
    if (lane == 0) {
      T* di = static_cast<T*>(a.dinit) + b * a.dis_b + ra * a.dis_c;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        float2 acc = f2(0.f, 0.f);
#pragma unroll
        for (int kk = 0; kk <= i; ++kk) acc = fma2(wp[kk], dq[i - kk], acc);
        if (fa != nullptr && i - L >= 0) {
          if (va) acc.x += Cvt<T>::f(fa[(i - L) * a.fs_l]);
          if (vb) acc.y += Cvt<T>::f(fa[a.fs_c + (i - L) * a.fs_l]);
        }
        if (va) di[i * a.dis_l] = Cvt<T>::to(acc.x);
        if (vb) di[a.dis_c + i * a.dis_l] = Cvt<T>::to(acc.y);
      }
    }
  }

  float2 dw[W];
#pragma unroll
  for (int k = 0; k < W; ++k) dw[k] = f2(0.f, 0.f);
  float2 db = f2(0.f, 0.f);
  const bool owner = lane < 31;

  for (int k = 0; k < ntiles; ++k) {
    const unsigned s = k % NS, use = k / NS;
    if (!mbar_wait(&full[s], use & 1)) return;
    const unsigned t = (unsigned)(t0 + k * kBwdStep);
    unsigned char* rowa = smem + s * SB + (2 * warp) * RB + ((ba + t) & inm) * sizeof(T);
    unsigned char* rowb = smem + s * SB + (2 * warp + 1) * RB + ((bb + t) & inm) * sizeof(T);
    if (t0 == 0 && k == 0) {
      if (lane == 0) {
        if (va) fix_row_head<T>(rowa, off_a, ir, a.is_l, H);
        if (vb) fix_row_head<T>(rowb, off_b, ir != nullptr ? ir + a.is_c : nullptr, a.is_l, H);
        fence_proxy_async_smem();
      }
      __syncwarp();
    }
    float xa[8], xb[8], ga[8], gb[8];
    lds8_row<T>(rowa, lane, xa);
    lds8_row<T>(rowb, lane, xb);
    lds8_row<T>(rowa + TB, lane, ga);
    lds8_row<T>(rowb + TB, lane, gb);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const int qa = qa0 + k * kBwdStep, qb = qb0 + k * kBwdStep;
    float2 xp[8], d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xp[i] = f2(xa[i], xb[i]);
    float2 h[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const float2 up = shfl_up2(xp[8 - H + j], 1);
      const float2 nc = shfl2(xp[8 - H + j], 31 - 1);
      h[j] = lane == 0 ? carry[j] : up;
      carry[j] = nc;
    }
    const bool edge = qa < 0 || qb < 0 || qa + 8 > L || qb + 8 > L;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 pre = bp;
#pragma unroll
      for (int kk = 0; kk < W; ++kk) {
        const int q = i - H + kk;
        pre = fma2(wp[kk], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], pre);
      }
      const float2 g = f2(ga[i], gb[i]);
      d[i] = SILU ? mul2(g, silu_grad2(pre)) : g;
      if (edge) {
        // Outside the row: the neighbouring rows' elements carry no gradient.
        if (qa + i < 0 || qa + i >= L) d[i].x = 0.f;
        if (qb + i < 0 || qb + i >= L) d[i].y = 0.f;
      }
      if (owner) {
        db = add2(db, d[i]);
#pragma unroll
        for (int kk = 0; kk < W; ++kk) {
          const int q = i - H + kk;
          dw[kk] = fma2(d[i], q >= 0 ? xp[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H], dw[kk]);
        }
      }
    }
    // dx of this tile: the right halo of lane l is lane l + 1's first dpre.
    float2 rh[H];
#pragma unroll
    for (int j = 0; j < H; ++j) rh[j] = shfl_down2(d[j], 1);
    emit_dx_shift<T, W>(d, rh, wp, qa, qb, L, a, dxa, fa, va && owner, vb && owner);
  }
  // Warp sums of the dweight / dbias partials; lane 0 writes this item's slot.
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
    for (int kk = 0; kk < W; ++kk) dw[kk] = add2(dw[kk], shfl_down2(dw[kk], off));
    db = add2(db, shfl_down2(db, off));
  }
  if (lane == 0) {
    float* pp = a.partials + ((b * a.nseg + seg) * a.D + ra) * (W + 1);
    if (va) {
#pragma unroll
      for (int kk = 0; kk < W; ++kk) pp[kk] = dw[kk].x;
      pp[W] = db.x;
    }
    if (vb) {
#pragma unroll
      for (int kk = 0; kk < W; ++kk) pp[W + 1 + kk] = dw[kk].y;
      pp[2 * W + 1] = db.y;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

template <typename T>
CUtensorMapDataType tma_dtype() {
  if (sizeof(T) == 4) return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (std::is_same<T, __half>::value) return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 3-D map over the (L, D, B) view of a seqlen-contiguous tensor; box
// (256 positions, 8 channels, 1), zero fill outside.
template <typename T>
bool make_seq_map(CUtensorMap* m, const void* base, i64 L, i64 D, i64 B, i64 s_c, i64 s_b) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  const i64 esz = sizeof(T);
  if (D == 1) s_c = L;
  if (B == 1) s_b = D * s_c;
  cuuint64_t dims[3] = {(cuuint64_t)L, (cuuint64_t)D, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(s_c * esz), (cuuint64_t)(s_b * esz)};
  cuuint32_t box[3] = {(cuuint32_t)kTL, (cuuint32_t)kRows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, tma_dtype<T>(), 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_error_detail("cuTensorMapEncodeTiled returned %d (dims %llu,%llu,%llu strides %llu,%llu)", (int)r,
                     (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
                     (unsigned long long)strides[0], (unsigned long long)strides[1]);
  return r == CUDA_SUCCESS;
}

bool aligned_to(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0; }

// Unit seqlen stride, 16-byte aligned base and channel / batch pitches.
bool seq_tensor_ok(const void* base, i64 s_c, i64 s_l, i64 s_b, i64 B, i64 D, int esz) {
  return base != nullptr && s_l == 1 && aligned_to(base, 16) && (D == 1 || ((s_c * esz) % 16 == 0 && s_c > 0)) &&
         (B == 1 || ((s_b * esz) % 16 == 0 && s_b > 0)) && (s_c * esz) < (1LL << 40) && (s_b * esz) < (1LL << 40);
}

// 3-D map over seq_idx viewed as (L, 1, B) int32; box (256, 1, 1), zero
// fill past the end (only positions past L read it; their outputs are not
// stored and their dout is zero-filled too).
bool make_ids_map(CUtensorMap* m, const int* base, i64 L, i64 B, i64 s_b) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  if (B == 1) s_b = L;
  cuuint64_t dims[3] = {(cuuint64_t)L, 1, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(L * 4), (cuuint64_t)(s_b * 4)};
  cuuint32_t box[3] = {(cuuint32_t)kTL, 1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, const_cast<int*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_error_detail("cuTensorMapEncodeTiled returned %d for seq_idx (L %lld, B %lld)", (int)r, (long long)L,
                     (long long)B);
  return r == CUDA_SUCCESS;
}

// seq_idx that the id tiles can stream: unit position stride, 16-byte
// aligned rows.
// The sequence masks as (L, 1, B) uint16 with row pitch mask_pitch(L); box
// (256, 1, 1), zero fill past L (a zero mask gates every tap).
bool make_mask_map(CUtensorMap* m, const uint16_t* base, i64 L, i64 B) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  const i64 pitch = mask_pitch(L) * (i64)sizeof(uint16_t);
  cuuint64_t dims[3] = {(cuuint64_t)L, 1, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)pitch, (cuuint64_t)pitch};
  cuuint32_t box[3] = {(cuuint32_t)kTL, 1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_error_detail("cuTensorMapEncodeTiled returned %d for the sequence masks (L %lld, B %lld)", (int)r,
                     (long long)L, (long long)B);
  return r == CUDA_SUCCESS;
}

// Bytes of the sequence masks and their place in the workspace (after the
// partials, 256-byte aligned; the plan's aux_bytes).
i64 mask_bytes(i64 B, i64 L) { return B * mask_pitch(L) * (i64)sizeof(uint16_t); }
uint16_t* mask_buffer(const BwdArgs& a, const Plan& plan, int W) {
  const i64 partials = plan.n_partials * a.D * (i64)(W + 1) * (i64)sizeof(float);
  return reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(a.partials) + (partials + 255) / 256 * 256);
}

cudaError_t launch_seq_mask(const BwdArgs& a, int H, uint16_t* mask, cudaStream_t stream) {
  const i64 blocks = ceil_div(mask_pitch(a.L), (i64)256);
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const dim3 grid((unsigned)blocks, (unsigned)std::min<i64>(a.B, 65535));
  return launch_pdl(seq_mask_kernel, grid, dim3(256), 0, stream, a.seq, a.ss_b, a.ss_l, a.B, a.L, H, mask);
}

bool ids_ok(const int* seq, i64 s_l, i64 s_b, i64 B, i64 L) {
  return seq != nullptr && s_l == 1 && aligned_to(seq, 16) && (B == 1 || (s_b >= L && (s_b * 4) % 16 == 0)) &&
         (s_b * 4) < (1LL << 40);
}

bool seq_shape_ok(i64 B, i64 D, i64 L) {
  return B >= 1 && D >= 1 && L >= 8 && L % 8 == 0 && L < (1LL << 31) && D < (1LL << 31) && B < (1LL << 31);
}

// Elements from the base of a (B, D, L) tensor with unit seqlen stride to
// the end of its last row.
i64 sh_extent(i64 B, i64 D, i64 L, i64 s_c, i64 s_b) { return (B - 1) * s_b + (D - 1) * s_c + L; }

// View-row geometry for a tensor extent: rows of the largest power of two
// elements, 16 .. kShMaxRowBytes bytes, that divides the extent (sh_ok
// guarantees 16 bytes does); and the tile counts of the segments.
template <typename T>
ShiftGeom sh_geom(i64 extent, i64 L, i64 nseg, i64 seg_len, i64 step) {
  ShiftGeom g;
  g.tiles_full = (int)(seg_len / step);
  g.tiles_last = (int)ceil_div(L - (nseg - 1) * seg_len + unit_elems<T>() - 1, step);
  int in = kShMaxRowBytes / (int)sizeof(T);
  while (in > unit_elems<T>() && extent % in != 0) in >>= 1;
  g.in = in;
  g.in_log2 = 0;
  while ((1 << g.in_log2) < in) ++g.in_log2;
  g.rows = kTL / in + 1;
  g.tx = (unsigned)(kRows * g.rows * in * (int)sizeof(T));
  return g;
}

// The tensor as (in, extent / in, 1) view rows; box (in, kTL / in + 1, 1).
template <typename T>
bool make_sh_map(CUtensorMap* m, const void* base, i64 extent, const ShiftGeom& g) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  const i64 units = extent / g.in;
  const i64 rb = (i64)g.in * (i64)sizeof(T);
  cuuint64_t dims[3] = {(cuuint64_t)g.in, (cuuint64_t)units, 1};
  cuuint64_t strides[2] = {(cuuint64_t)rb, (cuuint64_t)(units * rb)};
  cuuint32_t box[3] = {(cuuint32_t)g.in, (cuuint32_t)g.rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, tma_dtype<T>(), 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_error_detail("cuTensorMapEncodeTiled returned %d (shifted rows, %lld view rows)", (int)r, (long long)units);
  return r == CUDA_SUCCESS;
}

// Rows with unit seqlen stride, every tensor 16-byte aligned, with the SAME
// strides (so one offset per row serves all of them), non-overlapping rows,
// and an extent that is a whole number of 16-byte units addressable by
// 32-bit view-row indices.
bool sh_ok(const void* base, i64 s_c, i64 s_l, i64 s_b, i64 B, i64 D, i64 L, int esz) {
  const i64 E = 16 / esz;
  const i64 ext = sh_extent(B, D, L, s_c, s_b);
  return base != nullptr && s_l == 1 && aligned_to(base, 16) && (D == 1 || s_c >= L) &&
         (B == 1 || s_b >= (D - 1) * s_c + L) && ext % E == 0 && (ext + 8 * s_c + 2 * kTL) / E < (1LL << 31);
}

// Shifted tiles: any L >= 8 (stores are masked at the row end); positions
// (-8 .. L + 2 tiles) are 32-bit in the kernels.
bool sh_shape_ok(i64 B, i64 D, i64 L) {
  return B >= 1 && D >= 1 && L >= 8 && L < (1LL << 31) - 4096 && D < (1LL << 31) && B < (1LL << 31);
}

// The shifted kernels take rows the 3-D maps cannot describe, without
// seq_idx (those take the register kernels).
bool fwd_shifted(size_t esz, const FwdArgs& a) {
  const int e = (int)esz;
  if (a.seq != nullptr || !sh_shape_ok(a.B, a.D, a.L)) return false;
  if (seq_shape_ok(a.B, a.D, a.L) && seq_tensor_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, e) &&
      seq_tensor_ok(a.out, a.os_c, a.os_l, a.os_b, a.B, a.D, e))
    return false;  // the 3-D maps apply
  return a.os_c == a.xs_c && a.os_b == a.xs_b && sh_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, a.L, e) &&
         sh_ok(a.out, a.os_c, a.os_l, a.os_b, a.B, a.D, a.L, e);
}

bool bwd_shifted(size_t esz, const BwdArgs& a) {
  const int e = (int)esz;
  if (a.seq != nullptr || !sh_shape_ok(a.B, a.D, a.L)) return false;
  if (seq_shape_ok(a.B, a.D, a.L) && seq_tensor_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, e) &&
      seq_tensor_ok(a.dout, a.gs_c, a.gs_l, a.gs_b, a.B, a.D, e) &&
      seq_tensor_ok(a.dx, a.dxs_c, a.dxs_l, a.dxs_b, a.B, a.D, e))
    return false;
  return a.gs_c == a.xs_c && a.gs_b == a.xs_b && a.dxs_c == a.xs_c && a.dxs_b == a.xs_b &&
         sh_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, a.L, e) && sh_ok(a.dout, a.gs_c, a.gs_l, a.gs_b, a.B, a.D, a.L, e) &&
         sh_ok(a.dx, a.dxs_c, a.dxs_l, a.dxs_b, a.B, a.D, a.L, e);
}

int esize(int dtype) { return dtype == 2 ? 4 : 2; }

template <typename K>
cudaError_t prepare(K kernel, size_t smem, std::atomic<uint64_t>& attr_done, std::atomic<int>& occ, int* nb) {
  // The shared-memory limit is a per-device (per-context) attribute: one
  // bit per device that has it set.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
  if (bit == 0 || !(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  return blocks_per_sm(kernel, kThreadsSeq, smem, occ, nb);
}

// Items = (batch, group of 8 channels, segment); segments split long rows
// when there are too few (batch, group) pairs to fill the GPU.  The launch
// runs ceil(items / resident blocks) waves, each as long as a segment's
// tiles plus a block's fixed start (barriers, weights, the halo and tail
// loads, the pipeline fill: about kStartTiles tiles), so the segment count
// minimises waves x (tiles per segment + kStartTiles).  One row of 256 tiles
// over 512 pairs with 444 resident blocks: 2 segments run 2.3 waves (the
// last a third full), 6 segments 6.9 waves.
#ifndef CC1D_SEQ_START_TILES
#define CC1D_SEQ_START_TILES 3
#endif
constexpr i64 kStartTiles = CC1D_SEQ_START_TILES;
constexpr i64 kMaxSegs = 4096;  // bounds the host search

// `step`: positions a tile advances (kTL, or kBwdStep for the overlapping
// backward tiles); segments are whole numbers of steps.
void seq_schedule(const DeviceInfo& dev, int nb, i64 B, i64 D, i64 L, i64 step, Plan* plan) {
  const i64 groups = ceil_div(D, (i64)kRows);
  const i64 pairs = B * groups;
  const i64 resident = std::max<i64>(1, (i64)dev.sms * nb);
  const i64 row_tiles = std::max<i64>(1, ceil_div(L, step));
  i64 seg_tiles = row_tiles;
  double best = -1.0;
  for (i64 n = 1; n <= std::min(row_tiles, kMaxSegs); ++n) {
    const i64 st = ceil_div(row_tiles, n);
    const double cost = (double)ceil_div(pairs * ceil_div(row_tiles, st), resident) * (double)(st + kStartTiles);
    if (best < 0.0 || cost < best) {
      best = cost;
      seg_tiles = st;
    }
    if (pairs * n >= 64 * resident) break;  // many waves already: splitting only adds starts
  }
  const i64 seg_len = seg_tiles * step;
  const i64 nseg = ceil_div(L, seg_len);
  plan->layout = kSeq;
  plan->vec = true;
  plan->threads = kThreadsSeq;
  plan->groups = groups;
  plan->nseg = nseg;
  plan->seg_len = seg_len;
  plan->n_items = pairs * nseg;
  plan->grid = pairs * nseg;
  plan->n_partials = B * nseg;
}

template <typename T, int W, bool HAS_SEQ, bool SILU>
cudaError_t seq_fwd_instance(SeqFwdParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem = (size_t)seq_fwd_stages<T>() * (seq_tile_bytes<T>() + (HAS_SEQ ? kIdsBytes : 0u)) +
                          2 * seq_fwd_stages<T>() * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(fwd_seq_tma_kernel<T, W, HAS_SEQ, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(fwd_seq_tma_kernel<T, W, HAS_SEQ, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsSeq), smem,
                    stream, *prm);
}

template <typename T, int W, bool HAS_SEQ, bool SILU>
cudaError_t seq_bwd_instance(SeqBwdParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem = (size_t)seq_bwd_stages<T>() * (2 * seq_tile_bytes<T>() + (HAS_SEQ ? kMaskBytes : 0u)) +
                          2 * seq_bwd_stages<T>() * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(bwd_seq_tma_kernel<T, W, HAS_SEQ, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(bwd_seq_tma_kernel<T, W, HAS_SEQ, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsSeq), smem,
                    stream, *prm);
}

template <typename T, int W, bool SILU>
cudaError_t shift_fwd_instance(SeqFwdParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem =
      (size_t)seq_fwd_stages<T>() * kRows * sh_row_bytes<T>() + 2 * seq_fwd_stages<T>() * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(fwd_shift_tma_kernel<T, W, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(fwd_shift_tma_kernel<T, W, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsSeq), smem, stream,
                    *prm);
}

template <typename T, int W, bool SILU>
cudaError_t shift_bwd_instance(SeqBwdParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem =
      (size_t)seq_bwd_stages<T>() * 2 * kRows * sh_row_bytes<T>() + 2 * seq_bwd_stages<T>() * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(bwd_shift_tma_kernel<T, W, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(bwd_shift_tma_kernel<T, W, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsSeq), smem, stream,
                    *prm);
}

struct SeqFwdOp {
  const FwdArgs& a;
  Plan* plan;
  cudaStream_t stream;
  bool launch;
  template <typename T, int W>
  cudaError_t operator()() {
    const bool silu = a.silu != 0;
    const bool sh = fwd_shifted(sizeof(T), a);
    SeqFwdParams* prm = nullptr;
    SeqFwdParams storage;
    if (launch) {
      storage.a = a;
      storage.a.nseg = plan->nseg;
      storage.a.seg_len = plan->seg_len;
      storage.groups = plan->groups;
      const i64 ext = sh_extent(a.B, a.D, a.L, a.xs_c, a.xs_b);
      storage.sg = sh_geom<T>(ext, a.L, plan->nseg, plan->seg_len, kTL);
      const bool ok = sh ? make_sh_map<T>(&storage.map_x, a.x, ext, storage.sg)
                         : make_seq_map<T>(&storage.map_x, a.x, a.L, a.D, a.B, a.xs_c, a.xs_b);
      if (!ok) return cudaErrorInvalidValue;
      if (a.seq != nullptr && !make_ids_map(&storage.map_s, a.seq, a.L, a.B, a.ss_b)) return cudaErrorInvalidValue;
      prm = &storage;
    }
    int nb = 1;
    cudaError_t e;
    if (sh)
      e = silu ? shift_fwd_instance<T, W, true>(prm, plan, stream, &nb)
               : shift_fwd_instance<T, W, false>(prm, plan, stream, &nb);
    else if (a.seq != nullptr)
      e = silu ? seq_fwd_instance<T, W, true, true>(prm, plan, stream, &nb)
               : seq_fwd_instance<T, W, true, false>(prm, plan, stream, &nb);
    else
      e = silu ? seq_fwd_instance<T, W, false, true>(prm, plan, stream, &nb)
               : seq_fwd_instance<T, W, false, false>(prm, plan, stream, &nb);
    if (e != cudaSuccess || launch) return e;
    DeviceInfo dev;
    e = device_info(&dev);
    if (e != cudaSuccess) return e;
    seq_schedule(dev, nb, a.B, a.D, a.L, kTL, plan);
    plan->n_partials = 0;
    plan->aux_bytes = 0;
    return cudaSuccess;
  }
};

struct SeqBwdOp {
  const BwdArgs& a;
  Plan* plan;
  cudaStream_t stream;
  bool launch;
  template <typename T, int W>
  cudaError_t operator()() {
    const bool silu = a.silu != 0;
    const bool sh = bwd_shifted(sizeof(T), a);
    SeqBwdParams* prm = nullptr;
    SeqBwdParams storage;
    if (launch) {
      storage.a = a;
      storage.a.nseg = plan->nseg;
      storage.a.seg_len = plan->seg_len;
      storage.groups = plan->groups;
      const i64 ext = sh_extent(a.B, a.D, a.L, a.xs_c, a.xs_b);
      storage.sg = sh_geom<T>(ext, a.L, plan->nseg, plan->seg_len, kBwdStep);
      const bool ok = sh ? (make_sh_map<T>(&storage.map_x, a.x, ext, storage.sg) &&
                            make_sh_map<T>(&storage.map_g, a.dout, ext, storage.sg))
                         : (make_seq_map<T>(&storage.map_x, a.x, a.L, a.D, a.B, a.xs_c, a.xs_b) &&
                            make_seq_map<T>(&storage.map_g, a.dout, a.L, a.D, a.B, a.gs_c, a.gs_b));
      if (!ok) return cudaErrorInvalidValue;
      if (a.seq != nullptr) {
        // The backward reads sequence masks, written just before it.
        uint16_t* mask = mask_buffer(a, *plan, W);
        if (!make_mask_map(&storage.map_s, mask, a.L, a.B)) return cudaErrorInvalidValue;
        const cudaError_t em = launch_seq_mask(a, W - 1, mask, stream);
        if (em != cudaSuccess) return em;
      }
      prm = &storage;
    }
    int nb = 1;
    cudaError_t e;
    if (sh)
      e = silu ? shift_bwd_instance<T, W, true>(prm, plan, stream, &nb)
               : shift_bwd_instance<T, W, false>(prm, plan, stream, &nb);
    else if (a.seq != nullptr)
      e = silu ? seq_bwd_instance<T, W, true, true>(prm, plan, stream, &nb)
               : seq_bwd_instance<T, W, true, false>(prm, plan, stream, &nb);
    else
      e = silu ? seq_bwd_instance<T, W, false, true>(prm, plan, stream, &nb)
               : seq_bwd_instance<T, W, false, false>(prm, plan, stream, &nb);
    if (e != cudaSuccess || launch) return e;
    DeviceInfo dev;
    e = device_info(&dev);
    if (e != cudaSuccess) return e;
    seq_schedule(dev, nb, a.B, a.D, a.L, kBwdStep, plan);
    plan->aux_bytes = (!sh && a.seq != nullptr) ? mask_bytes(a.B, a.L) : 0;
    return cudaSuccess;
  }
};

}  // namespace

bool fwd_seq_tma_eligible(int dtype, const FwdArgs& a) {
  const int esz = esize(dtype);
  if (encode_fn() != nullptr && fwd_shifted((size_t)esz, a)) return true;
  return (a.seq == nullptr || ids_ok(a.seq, a.ss_l, a.ss_b, a.B, a.L)) && seq_shape_ok(a.B, a.D, a.L) &&
         encode_fn() != nullptr &&
         seq_tensor_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, esz) &&
         seq_tensor_ok(a.out, a.os_c, a.os_l, a.os_b, a.B, a.D, esz);
}

bool bwd_seq_tma_eligible(int dtype, const BwdArgs& a) {
  const int esz = esize(dtype);
  if (encode_fn() != nullptr && bwd_shifted((size_t)esz, a)) return true;
  return (a.seq == nullptr || ids_ok(a.seq, a.ss_l, a.ss_b, a.B, a.L)) && seq_shape_ok(a.B, a.D, a.L) &&
         encode_fn() != nullptr &&
         seq_tensor_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, a.D, esz) &&
         seq_tensor_ok(a.dout, a.gs_c, a.gs_l, a.gs_b, a.B, a.D, esz) &&
         seq_tensor_ok(a.dx, a.dxs_c, a.dxs_l, a.dxs_b, a.B, a.D, esz);
}

cudaError_t plan_fwd_seq_tma(int dtype, int width, const FwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, SeqFwdOp{a, plan, nullptr, false});
}

cudaError_t launch_fwd_seq_tma(int dtype, int width, const FwdArgs& a, const Plan& plan, cudaStream_t stream) {
  Plan p = plan;
  return dispatch(dtype, width, SeqFwdOp{a, &p, stream, true});
}

cudaError_t plan_bwd_seq_tma(int dtype, int width, const BwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, SeqBwdOp{a, plan, nullptr, false});
}

cudaError_t launch_bwd_seq_tma(int dtype, int width, const BwdArgs& a, const Plan& plan, cudaStream_t stream) {
  Plan p = plan;
  return dispatch(dtype, width, SeqBwdOp{a, &p, stream, true});
}

cudaError_t read_seq_wait_timeouts(unsigned* count) { return tu_read_wait_timeouts(count); }

}  // namespace cc1d
