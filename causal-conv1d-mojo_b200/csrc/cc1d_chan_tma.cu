// Channel-last (dim is the unit-stride axis, the Mamba layout) forward and
// backward kernels, fed by a TMA pipeline.  sm_100a.
//
// Block = 4 consumer warps + 1 producer warp, owning a group of 256
// channels and a contiguous range of (b, t) rows of it.  The producer's
// elected lane streams [TR rows x 256 channels] tiles of x (and grad_out in
// the backward) with cp.async.bulk.tensor.3d into a 4-stage shared-memory
// ring; full/empty mbarriers hand stages back and forth.  Each consumer
// thread owns 2 adjacent channels, walks the rows in order keeping the last
// W-1 rows in registers (so the causal halo is read once per run), computes
// with packed fp32 (sm_100 FFMA2) and stores 2 outputs per row as one
// 4-byte word (a warp writes 128 contiguous bytes per row).
//
// Forward:  out[t] = act(bias + sum_k w[k] * xc[t-(W-1)+k])
// Backward: dpre[t] = dout[t] * silu'(pre[t]); dx[p] = sum_j w[W-1-j] *
//           dpre[p+j] emitted W-1 rows after p; dweight/dbias partial sums
//           per thread, written once per block to the workspace (reduced in
//           fixed order by finalize_kernel in cc1d_bwd.cu).
// Semantics are those of cc1d_fwd.cu / cc1d_bwd.cu (reference CPU kernels
// src/causal_conv1d_mojo/fwd_cpu/kernel.mojo:64-117 and
// bwd_full_cpu/kernel.mojo:26-314, final/initial states as
// src/causal_conv1d_mojo/reference.py:50-56).
#include <cudaTypedefs.h>

#include <type_traits>

#include "cc1d_dispatch.cuh"
#include "cc1d_tma.cuh"

namespace cc1d {

namespace {

// Pipeline shape.  The defaults were the fastest of a sweep of stage sizes,
// stage counts and occupancy bounds measured on B200 at the Mamba-2 prefill
// shape; overridable with -D for tuning sweeps.
#ifndef CC1D_FWD_STAGE_BYTES
#define CC1D_FWD_STAGE_BYTES 8192
#endif
#ifndef CC1D_FWD_STAGES
#define CC1D_FWD_STAGES 4
#endif
#ifndef CC1D_FWD_MIN_BLOCKS
#define CC1D_FWD_MIN_BLOCKS 6
#endif
#ifndef CC1D_BWD_TILE_BYTES
#define CC1D_BWD_TILE_BYTES 8192
#endif
#ifndef CC1D_BWD_STAGES
#define CC1D_BWD_STAGES 3
#endif
#ifndef CC1D_BWD_MIN_BLOCKS
#define CC1D_BWD_MIN_BLOCKS 3
#endif

constexpr int kCW = 4;                 // consumer warps
constexpr int kGroup = kCW * 32 * 2;   // channels per block
constexpr int kFwdStages = CC1D_FWD_STAGES;
constexpr int kBwdStages = CC1D_BWD_STAGES;
constexpr int kThreadsTma = (kCW + 1) * 32;

// Rows per pipeline stage (forward: x; backward: x and grad_out each).
template <typename T>
constexpr int fwd_rows() {
  return CC1D_FWD_STAGE_BYTES / (kGroup * (int)sizeof(T));
}
template <typename T>
constexpr int bwd_rows() {
  return CC1D_BWD_TILE_BYTES / (kGroup * (int)sizeof(T));
}

struct alignas(64) FwdTmaParams {
  CUtensorMap map_x;
  FwdArgs a;
};
struct alignas(64) BwdTmaParams {
  CUtensorMap map_x;
  CUtensorMap map_g;
  BwdArgs a;
};

template <typename T>
__device__ __forceinline__ float2 load_pair(const T* p) {
  return Pair<T>::unpack(*reinterpret_cast<const typename Pair<T>::W*>(p));
}

template <typename T>
__device__ __forceinline__ float2 load_pair_strided(const T* p, i64 stride) {
  return f2(Cvt<T>::f(p[0]), Cvt<T>::f(p[stride]));
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

template <typename T, int W, bool HAS_SEQ, bool SILU>
__global__ void __launch_bounds__(kThreadsTma, CC1D_FWD_MIN_BLOCKS) fwd_chan_tma_kernel(const __grid_constant__ FwdTmaParams p) {
  typedef Pair<T> P;
  typedef typename P::W PW;
  constexpr int H = W - 1;
  constexpr int TR = fwd_rows<T>();
  constexpr int ROW_WORDS = kGroup / 2;
  constexpr unsigned STAGE_BYTES = TR * kGroup * sizeof(T);
  static_assert(TR <= 32, "seq ids of a tile are held one per lane");
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kFwdStages * STAGE_BYTES);
  uint64_t* empty = full + kFwdStages;
  const FwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 grp = blockIdx.x / a.splits;
  const i64 split = blockIdx.x - grp * a.splits;
  const i64 c0 = grp * kGroup;
  const i64 R = a.B * a.L;
  const i64 cr0 = split * a.rows_per_split;
  const i64 cr1 = min(R, cr0 + a.rows_per_split);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // inputs of this launch may come from the previous kernel
  griddep_launch_dependents();

  if (warp == kCW) {
    // Producer: one elected lane issues every tile of this block.
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      unsigned k = 0;
      bool live = true;
      for (i64 r = cr0; r < cr1 && live;) {
        const i64 b = r / a.L;
        const i64 t0 = r - b * a.L;
        const i64 t1 = min(a.L, t0 + (cr1 - r));
        r += t1 - t0;
        for (i64 t = t0; t < t1; t += TR, ++k) {
          const unsigned s = k % kFwdStages, use = k / kFwdStages;
          if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
            live = false;  // consumers stopped: issue nothing more
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_3d(smem + s * STAGE_BYTES, &p.map_x, &full[s], (int)c0, (int)t, (int)b);
        }
      }
      mbar_drain(full, k, kFwdStages);
    }
    return;
  }

  const int tid = threadIdx.x;  // 0 .. 127
  const i64 c = c0 + 2 * tid;
  const bool valid = c < a.D;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ out = static_cast<T*>(a.out);
  T* __restrict__ fin = static_cast<T*>(a.fin);

  float2 wv[W];
#pragma unroll
  for (int k = 0; k < W; ++k)
    wv[k] = valid ? load_pair_strided(wt + c * a.ws_c + k * a.ws_k, a.ws_c) : f2(0.f, 0.f);
  const float2 bv = (bias && valid) ? load_pair_strided(bias + c * a.bs, a.bs) : f2(0.f, 0.f);

  unsigned k = 0;
  for (i64 r = cr0; r < cr1;) {
    const i64 b = r / a.L;
    const i64 t0 = r - b * a.L;
    const i64 t1 = min(a.L, t0 + (cr1 - r));
    r += t1 - t0;
    // Window: xc at positions t0-H .. t0-1.
    float2 xw[H];
    int sw[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const i64 q = t0 - H + j;
      xw[j] = f2(0.f, 0.f);
      sw[j] = kNoSeq;
      if (q >= 0) {
        if (valid) xw[j] = load_pair(x + b * a.xs_b + q * a.xs_l + c);
        if (HAS_SEQ) sw[j] = seq[b * a.ss_b + q * a.ss_l];
      } else if (init && valid) {
        xw[j] = load_pair_strided(init + b * a.is_b + c * a.is_c + (q + H) * a.is_l, a.is_c);
      }
    }
    T* orow = out + b * a.os_b + t0 * a.os_l + c;
    for (i64 t = t0; t < t1; t += TR, ++k) {
      const unsigned s = k % kFwdStages, use = k / kFwdStages;
      if (!mbar_wait(&full[s], use & 1)) return;
      const PW* tile = reinterpret_cast<const PW*>(smem + s * STAGE_BYTES) + tid;
      int sreg = 0;
      if (HAS_SEQ) sreg = (t + lane < t1 && lane < TR) ? seq[b * a.ss_b + (t + lane) * a.ss_l] : kNoSeq;
      const int nr = (int)min((i64)TR, t1 - t);
      // With seq_idx, a tile whose rows and W-1 halo all carry the same
      // non-negative id (no sequence boundary, no padding) needs no gating.
      bool gate = HAS_SEQ;
      if (HAS_SEQ) {
        const int s0 = sw[0];
        bool same = s0 >= 0;
#pragma unroll
        for (int j = 1; j < H; ++j) same = same && sw[j] == s0;
        same = __all_sync(kFull, same && (lane >= nr || sreg == s0));
        if (same) {
          gate = false;
#pragma unroll
          for (int j = 0; j < H; ++j) sw[j] = s0;
        }
      }
      if (gate) {
#pragma unroll
        for (int rr = 0; rr < TR; ++rr) {
          if (rr >= nr) break;
          const float2 xv = P::unpack(tile[rr * ROW_WORDS]);
          const int sid = __shfl_sync(kFull, sreg, rr);
          float2 acc = bv;
#pragma unroll
          for (int j = 0; j < H; ++j)
            if (sw[j] == sid) acc = fma2(wv[j], xw[j], acc);
          acc = fma2(wv[H], xv, acc);
          if (SILU) acc = silu2(acc);
          if (sid < 0) acc = f2(0.f, 0.f);
          if (valid) *reinterpret_cast<PW*>(orow) = P::pack(acc);
          orow += a.os_l;
#pragma unroll
          for (int j = 0; j < H - 1; ++j) {
            xw[j] = xw[j + 1];
            sw[j] = sw[j + 1];
          }
          xw[H - 1] = xv;
          sw[H - 1] = sid;
        }
      } else if (nr == TR && valid) {
        // Full tile, in-range channels: no per-row checks; row addresses are
        // the tile's base plus compile-time multiples of the row pitch.
        const i64 pitch = a.os_l;
#pragma unroll
        for (int rr = 0; rr < TR; ++rr) {
          const float2 xv = P::unpack(tile[rr * ROW_WORDS]);
          float2 acc = bv;
#pragma unroll
          for (int j = 0; j < H; ++j) acc = fma2(wv[j], xw[j], acc);
          acc = fma2(wv[H], xv, acc);
          if (SILU) acc = silu2(acc);
          *reinterpret_cast<PW*>(orow + rr * pitch) = P::pack(acc);
#pragma unroll
          for (int j = 0; j < H - 1; ++j) xw[j] = xw[j + 1];
          xw[H - 1] = xv;
        }
        orow += TR * pitch;
      } else {
#pragma unroll
        for (int rr = 0; rr < TR; ++rr) {
          if (rr >= nr) break;
          const float2 xv = P::unpack(tile[rr * ROW_WORDS]);
          float2 acc = bv;
#pragma unroll
          for (int j = 0; j < H; ++j) acc = fma2(wv[j], xw[j], acc);
          acc = fma2(wv[H], xv, acc);
          if (SILU) acc = silu2(acc);
          if (valid) *reinterpret_cast<PW*>(orow) = P::pack(acc);
          orow += a.os_l;
#pragma unroll
          for (int j = 0; j < H - 1; ++j) xw[j] = xw[j + 1];
          xw[H - 1] = xv;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (fin != nullptr && t1 == a.L && valid) {
#pragma unroll
      for (int j = 0; j < H; ++j) {
        T* f = fin + b * a.fs_b + c * a.fs_c + j * a.fs_l;
        f[0] = Cvt<T>::to(xw[j].x);
        f[a.fs_c] = Cvt<T>::to(xw[j].y);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

template <typename T, int W>
struct BwdState {
  float2 wv[W];
  float2 bv;
  float2 xw[W - 1];  // xc at positions t-H .. t-1
  float2 pw[W - 1];          // dpre at positions t-H .. t-1
  int sw[W - 1];             // seq ids at positions t-H .. t-1
  float2 dwa[W];
  float2 dba;
};

// One time step t of the backward for a thread's 2 channels: recomputes
// dpre[t]; if `own`, accumulates dweight/dbias; if `emit`, writes dx (or
// dinitial_states) of position t-H.  CHECK=false is the interior path
// (own and emit known true, no states involved).
template <typename T, int W, bool HAS_SEQ, bool SILU, bool CHECK>
__device__ __forceinline__ void bwd_step(BwdState<T, W>& st, float2 xv, float2 gv, int sid, bool own,
                                         bool emit, T* dxrow, const BwdArgs& a, i64 b, i64 c, i64 p, bool valid) {
  constexpr int H = W - 1;
  typedef Pair<T> P;
  float2 pre = st.bv;
#pragma unroll
  for (int j = 0; j < H; ++j)
    if (!HAS_SEQ || st.sw[j] == sid) pre = fma2(st.wv[j], st.xw[j], pre);
  pre = fma2(st.wv[H], xv, pre);
  float2 g = SILU ? mul2(gv, silu_grad2(pre)) : gv;
  if (HAS_SEQ && sid < 0) g = f2(0.f, 0.f);
  if (!CHECK || own) {
    st.dba = add2(st.dba, g);
#pragma unroll
    for (int j = 0; j < H; ++j)
      if (!HAS_SEQ || st.sw[j] == sid) st.dwa[j] = fma2(g, st.xw[j], st.dwa[j]);
    st.dwa[H] = fma2(g, xv, st.dwa[H]);
  }
  if (!CHECK || emit) {
    const int sp = st.sw[0];
    float2 acc = f2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < H; ++j)
      if (!HAS_SEQ || st.sw[j] == sp) acc = fma2(st.wv[H - j], st.pw[j], acc);
    if (!HAS_SEQ || sid == sp) acc = fma2(st.wv[0], g, acc);
    if (CHECK) {
      if (a.dfin) {
        const i64 q = p + H - a.L;
        if (q >= 0 && valid)
          acc = add2(acc, load_pair_strided(static_cast<const T*>(a.dfin) + b * a.fs_b + c * a.fs_c + q * a.fs_l,
                                            a.fs_c));
      }
      if (valid) {
        if (p >= 0) {
          *reinterpret_cast<typename P::W*>(dxrow) = P::pack(acc);
        } else {
          T* d = static_cast<T*>(a.dinit) + b * a.dis_b + c * a.dis_c + (p + H) * a.dis_l;
          d[0] = Cvt<T>::to(acc.x);
          d[a.dis_c] = Cvt<T>::to(acc.y);
        }
      }
    } else if (valid) {
      *reinterpret_cast<typename P::W*>(dxrow) = P::pack(acc);
    }
  }
#pragma unroll
  for (int j = 0; j < H - 1; ++j) {
    st.xw[j] = st.xw[j + 1];
    st.pw[j] = st.pw[j + 1];
    st.sw[j] = st.sw[j + 1];
  }
  st.xw[H - 1] = xv;
  st.pw[H - 1] = g;
  st.sw[H - 1] = sid;
}

template <typename T, int W, bool HAS_SEQ, bool SILU>
__global__ void __launch_bounds__(kThreadsTma, CC1D_BWD_MIN_BLOCKS) bwd_chan_tma_kernel(const __grid_constant__ BwdTmaParams p) {
  typedef Pair<T> P;
  typedef typename P::W PW;
  constexpr int H = W - 1;
  constexpr int TR = bwd_rows<T>();
  constexpr int ROW_WORDS = kGroup / 2;
  constexpr unsigned TILE_BYTES = TR * kGroup * sizeof(T);
  constexpr unsigned STAGE_BYTES = 2 * TILE_BYTES;
  static_assert(TR <= 32, "seq ids of a tile are held one per lane");
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBwdStages * STAGE_BYTES);
  uint64_t* empty = full + kBwdStages;
  const BwdArgs& a = p.a;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const i64 grp = blockIdx.x / a.splits;
  const i64 split = blockIdx.x - grp * a.splits;
  const i64 c0 = grp * kGroup;
  const i64 R = a.B * a.L;
  const i64 cr0 = split * a.rows_per_split;
  const i64 cr1 = min(R, cr0 + a.rows_per_split);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // inputs of this launch may come from the previous kernel
  griddep_launch_dependents();

  if (warp == kCW) {
    if (lane == 0) {
      prefetch_tensormap(&p.map_x);
      prefetch_tensormap(&p.map_g);
      unsigned k = 0;
      bool live = true;
      for (i64 r = cr0; r < cr1 && live;) {
        const i64 b = r / a.L;
        const i64 t0 = r - b * a.L;
        const i64 t1 = min(a.L, t0 + (cr1 - r));
        r += t1 - t0;
        const i64 tl = min(a.L, t1 + H);  // dx of the last rows needs H rows more
        for (i64 t = t0; t < tl; t += TR, ++k) {
          const unsigned s = k % kBwdStages, use = k / kBwdStages;
          if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) {
            live = false;  // consumers stopped: issue nothing more
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          unsigned char* dst = smem + s * STAGE_BYTES;
          tma_load_3d(dst, &p.map_x, &full[s], (int)c0, (int)t, (int)b);
          tma_load_3d(dst + TILE_BYTES, &p.map_g, &full[s], (int)c0, (int)t, (int)b);
        }
      }
      mbar_drain(full, k, kBwdStages);
    }
    return;
  }

  const int tid = threadIdx.x;
  const i64 c = c0 + 2 * tid;
  const bool valid = c < a.D;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ dx = static_cast<T*>(a.dx);

  BwdState<T, W> st;
#pragma unroll
  for (int k = 0; k < W; ++k) {
    st.wv[k] = valid ? load_pair_strided(wt + c * a.ws_c + k * a.ws_k, a.ws_c) : f2(0.f, 0.f);
    st.dwa[k] = f2(0.f, 0.f);
  }
  st.bv = (bias && valid) ? load_pair_strided(bias + c * a.bs, a.bs) : f2(0.f, 0.f);
  st.dba = f2(0.f, 0.f);
  const bool has_dinit = a.dinit != nullptr;

  unsigned k = 0;
  for (i64 r = cr0; r < cr1;) {
    const i64 b = r / a.L;
    const i64 t0 = r - b * a.L;
    const i64 t1 = min(a.L, t0 + (cr1 - r));
    r += t1 - t0;
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const i64 q = t0 - H + j;
      st.xw[j] = f2(0.f, 0.f);
      st.pw[j] = f2(0.f, 0.f);
      st.sw[j] = kNoSeq;
      if (q >= 0) {
        if (valid) st.xw[j] = load_pair(x + b * a.xs_b + q * a.xs_l + c);
        if (HAS_SEQ) st.sw[j] = seq[b * a.ss_b + q * a.ss_l];
      } else if (init && valid) {
        st.xw[j] = load_pair_strided(init + b * a.is_b + c * a.is_c + (q + H) * a.is_l, a.is_c);
      }
    }
    const i64 tl = min(a.L, t1 + H);
    // dx row pointer of position t-H for the step at t.
    T* dxrow = dx + b * a.dxs_b + (t0 - H) * a.dxs_l + c;
    for (i64 t = t0; t < tl; t += TR, ++k) {
      const unsigned s = k % kBwdStages, use = k / kBwdStages;
      if (!mbar_wait(&full[s], use & 1)) return;
      const PW* tx = reinterpret_cast<const PW*>(smem + s * STAGE_BYTES) + tid;
      const PW* tg = reinterpret_cast<const PW*>(smem + s * STAGE_BYTES + TILE_BYTES) + tid;
      int sreg = 0;
      if (HAS_SEQ) sreg = (t + lane < tl && lane < TR) ? seq[b * a.ss_b + (t + lane) * a.ss_l] : kNoSeq;
      const int nr = (int)min((i64)TR, tl - t);
      // With seq_idx, a tile whose rows and W-1 halo all carry the same
      // non-negative id needs no gating (dx of its rows reads dpre of the
      // next W-1 rows, which are in this tile or gated by the later tiles'
      // own checks through the dpre window's ids).
      bool gate = HAS_SEQ;
      if (HAS_SEQ) {
        const int s0 = st.sw[0];
        bool same = s0 >= 0;
#pragma unroll
        for (int j = 1; j < H; ++j) same = same && st.sw[j] == s0;
        same = __all_sync(kFull, same && (lane >= nr || sreg == s0));
        if (same) gate = false;
      }
      if (!gate && nr == TR && t >= t0 + H && t + TR <= t1) {
        // Interior tile: every step owns its row and emits a dx row.
        const int s0 = HAS_SEQ ? st.sw[0] : 0;
#pragma unroll
        for (int rr = 0; rr < TR; ++rr) {
          bwd_step<T, W, false, SILU, false>(st, P::unpack(tx[rr * ROW_WORDS]), P::unpack(tg[rr * ROW_WORDS]), 0,
                                             true, true, dxrow, a, b, c, 0, valid);
          dxrow += a.dxs_l;
        }
        if (HAS_SEQ) {
#pragma unroll
          for (int j = 0; j < H; ++j) st.sw[j] = s0;
        }
      } else {
#pragma unroll
        for (int rr = 0; rr < TR; ++rr) {
          if (rr >= nr) break;
          const i64 tt = t + rr;
          const int sid = HAS_SEQ ? __shfl_sync(kFull, sreg, rr) : 0;
          const i64 pp = tt - H;
          const bool emit = pp >= t0 || (t0 == 0 && pp < 0 && has_dinit);
          bwd_step<T, W, HAS_SEQ, SILU, true>(st, P::unpack(tx[rr * ROW_WORDS]), P::unpack(tg[rr * ROW_WORDS]),
                                               sid, tt < t1, emit, dxrow, a, b, c, pp, valid);
          dxrow += a.dxs_l;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // Steps past the end of the sequence (no data; dpre = 0 there).
    for (i64 tt = max(tl, t0); tt < t1 + H; ++tt) {
      const i64 pp = tt - H;
      const bool emit = pp >= t0 || (t0 == 0 && pp < 0 && has_dinit);
      bwd_step<T, W, HAS_SEQ, SILU, true>(st, f2(0.f, 0.f), f2(0.f, 0.f), kNoSeq, false, emit, dxrow, a, b, c, pp,
                                           valid);
      dxrow += a.dxs_l;
    }
  }
  if (valid) {
    float* pp = a.partials + (split * a.D + c) * (W + 1);
#pragma unroll
    for (int j = 0; j < W; ++j) {
      pp[j] = st.dwa[j].x;
      pp[W + 1 + j] = st.dwa[j].y;
    }
    pp[W] = st.dba.x;
    pp[W + 1 + W] = st.dba.y;
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

// 3-D map over a channel-last (B, L, D) view: dims (D, L, B), box
// (kGroup, rows, 1), zero fill outside the tensor.
template <typename T>
bool make_map(CUtensorMap* m, const void* base, i64 D, i64 L, i64 B, i64 s_l, i64 s_b, int rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (enc == nullptr) return false;
  const i64 esz = sizeof(T);
  if (B == 1) s_b = L * s_l;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(s_l * esz), (cuuint64_t)(s_b * esz)};
  cuuint32_t box[3] = {(cuuint32_t)kGroup, (cuuint32_t)rows, 1};
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

// TMA source: unit channel stride, 16-byte aligned base and row/batch pitches.
bool tma_source_ok(const void* base, i64 s_c, i64 s_l, i64 s_b, i64 B, int esz) {
  return base != nullptr && s_c == 1 && aligned_to(base, 16) && (s_l * esz) % 16 == 0 && s_l > 0 &&
         (B == 1 || ((s_b * esz) % 16 == 0 && s_b > 0)) && (s_l * esz) < (1LL << 40) && (s_b * esz) < (1LL << 40);
}

// Pair store target: unit channel stride, 2-element aligned rows.
bool pair_dest_ok(const void* base, i64 s_c, i64 s_l, i64 s_b, int esz) {
  return base != nullptr && s_c == 1 && aligned_to(base, 2 * esz) && s_l % 2 == 0 && s_b % 2 == 0;
}

bool shape_ok(i64 B, i64 D, i64 L) {
  return B >= 1 && L >= 2 && D >= 2 && D % 2 == 0 && D < (1LL << 31) && L < (1LL << 31) && B < (1LL << 31);
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
  return blocks_per_sm(kernel, kThreadsTma, smem, occ, nb);
}

void split_rows(const DeviceInfo& dev, int nb, i64 D, i64 R, int tile_rows, Plan* plan) {
  const i64 groups = ceil_div(D, (i64)kGroup);
  const i64 target = (i64)dev.sms * nb;
  i64 splits = std::max<i64>(1, target / groups);
  i64 rps = std::max<i64>(ceil_div(R, splits), (i64)tile_rows);
  splits = ceil_div(R, rps);
  plan->layout = kChan;
  plan->vec = true;
  plan->threads = kThreadsTma;
  plan->groups = groups;
  plan->splits = splits;
  plan->rows_per_split = rps;
  plan->grid = groups * splits;
  plan->n_partials = splits;
}

template <typename T, int W, bool SEQ, bool SILU>
cudaError_t fwd_instance(FwdTmaParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem = (size_t)kFwdStages * fwd_rows<T>() * kGroup * sizeof(T) + 2 * kFwdStages * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(fwd_chan_tma_kernel<T, W, SEQ, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(fwd_chan_tma_kernel<T, W, SEQ, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsTma), smem, stream,
                    *prm);
}

template <typename T, int W, bool SEQ, bool SILU>
cudaError_t bwd_instance(BwdTmaParams* prm, const Plan* plan, cudaStream_t stream, int* nb_out) {
  constexpr size_t smem = (size_t)kBwdStages * 2 * bwd_rows<T>() * kGroup * sizeof(T) + 2 * kBwdStages * sizeof(uint64_t);
  static std::atomic<uint64_t> attr{0};
  static std::atomic<int> occ{0};
  int nb = 1;
  cudaError_t e = prepare(bwd_chan_tma_kernel<T, W, SEQ, SILU>, smem, attr, occ, &nb);
  if (e != cudaSuccess) return e;
  if (nb_out) *nb_out = nb;
  if (prm == nullptr) return cudaSuccess;
  return launch_pdl(bwd_chan_tma_kernel<T, W, SEQ, SILU>, dim3((unsigned)plan->grid), dim3(kThreadsTma), smem, stream,
                    *prm);
}

struct FwdTmaOp {
  const FwdArgs& a;
  Plan* plan;
  cudaStream_t stream;
  bool launch;
  template <typename T, int W>
  cudaError_t operator()() {
    const bool seq = a.seq != nullptr, silu = a.silu != 0;
    FwdTmaParams* prm = nullptr;
    FwdTmaParams storage;
    if (launch) {
      storage.a = a;
      storage.a.splits = plan->splits;
      storage.a.rows_per_split = plan->rows_per_split;
      if (!make_map<T>(&storage.map_x, a.x, a.D, a.L, a.B, a.xs_l, a.xs_b, fwd_rows<T>()))
        return cudaErrorInvalidValue;
      prm = &storage;
    }
    int nb = 1;
    cudaError_t e;
    if (seq)
      e = silu ? fwd_instance<T, W, true, true>(prm, plan, stream, &nb)
               : fwd_instance<T, W, true, false>(prm, plan, stream, &nb);
    else
      e = silu ? fwd_instance<T, W, false, true>(prm, plan, stream, &nb)
               : fwd_instance<T, W, false, false>(prm, plan, stream, &nb);
    if (e != cudaSuccess || launch) return e;
    DeviceInfo dev;
    e = device_info(&dev);
    if (e != cudaSuccess) return e;
    split_rows(dev, nb, a.D, a.B * a.L, fwd_rows<T>(), plan);
    plan->n_partials = 0;
    return cudaSuccess;
  }
};

struct BwdTmaOp {
  const BwdArgs& a;
  Plan* plan;
  cudaStream_t stream;
  bool launch;
  template <typename T, int W>
  cudaError_t operator()() {
    const bool seq = a.seq != nullptr, silu = a.silu != 0;
    BwdTmaParams* prm = nullptr;
    BwdTmaParams storage;
    if (launch) {
      storage.a = a;
      storage.a.splits = plan->splits;
      storage.a.rows_per_split = plan->rows_per_split;
      if (!make_map<T>(&storage.map_x, a.x, a.D, a.L, a.B, a.xs_l, a.xs_b, bwd_rows<T>()) ||
          !make_map<T>(&storage.map_g, a.dout, a.D, a.L, a.B, a.gs_l, a.gs_b, bwd_rows<T>()))
        return cudaErrorInvalidValue;
      prm = &storage;
    }
    int nb = 1;
    cudaError_t e;
    if (seq)
      e = silu ? bwd_instance<T, W, true, true>(prm, plan, stream, &nb)
               : bwd_instance<T, W, true, false>(prm, plan, stream, &nb);
    else
      e = silu ? bwd_instance<T, W, false, true>(prm, plan, stream, &nb)
               : bwd_instance<T, W, false, false>(prm, plan, stream, &nb);
    if (e != cudaSuccess || launch) return e;
    DeviceInfo dev;
    e = device_info(&dev);
    if (e != cudaSuccess) return e;
    split_rows(dev, nb, a.D, a.B * a.L, bwd_rows<T>(), plan);
    return cudaSuccess;
  }
};

}  // namespace

cudaError_t read_wait_timeouts(unsigned* count) {
  *count = 0;
  cudaError_t e = tu_read_wait_timeouts(count);
  if (e != cudaSuccess) return e;
  return read_seq_wait_timeouts(count);
}

bool fwd_tma_eligible(int dtype, const FwdArgs& a) {
  const int esz = esize(dtype);
  return shape_ok(a.B, a.D, a.L) && encode_fn() != nullptr &&
         tma_source_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, esz) &&
         pair_dest_ok(a.out, a.os_c, a.os_l, a.os_b, esz) && aligned_to(a.x, 2 * esz);
}

bool bwd_tma_eligible(int dtype, const BwdArgs& a) {
  const int esz = esize(dtype);
  return shape_ok(a.B, a.D, a.L) && encode_fn() != nullptr &&
         tma_source_ok(a.x, a.xs_c, a.xs_l, a.xs_b, a.B, esz) &&
         tma_source_ok(a.dout, a.gs_c, a.gs_l, a.gs_b, a.B, esz) &&
         pair_dest_ok(a.dx, a.dxs_c, a.dxs_l, a.dxs_b, esz);
}

cudaError_t plan_fwd_tma(int dtype, int width, const FwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, FwdTmaOp{a, plan, nullptr, false});
}

cudaError_t launch_fwd_tma(int dtype, int width, const FwdArgs& a, const Plan& plan, cudaStream_t stream) {
  Plan p = plan;
  return dispatch(dtype, width, FwdTmaOp{a, &p, stream, true});
}

cudaError_t plan_bwd_tma(int dtype, int width, const BwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, BwdTmaOp{a, plan, nullptr, false});
}

cudaError_t launch_bwd_tma(int dtype, int width, const BwdArgs& a, const Plan& plan, cudaStream_t stream) {
  Plan p = plan;
  return dispatch(dtype, width, BwdTmaOp{a, &p, stream, true});
}

}  // namespace cc1d
