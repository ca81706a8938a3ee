// Fused backward kernels of causal_conv1d_fn for sm_100a.
//
// With xc = cat([initial_states or 0, x]) and pre the recomputed
// pre-activation:
//   dpre[t]   = dout[t] * silu'(pre[t])      (dout[t] without activation;
//                                             0 where seq_idx[t] < 0)
//   dx[p]     = sum_{j<W} w[W-1-j] * dpre[p+j]           (p in [0, L))
//   dinit[i]  = the same sum at p = i-(W-1)               (i in [0, W-1))
//   dw[k]    += dpre[t] * xc[t-(W-1)+k]
//   dbias    += dpre[t]
// seq_idx gates each term on equal sequence ids, exactly as the forward.
// dfinal_states[q] (gradient of final_states = xc[L : L+W-1]) is added to
// the dx / dinit element at p = q + L - (W-1).
// Semantics follow the reference CPU kernel
// (src/causal_conv1d_mojo/bwd_full_cpu/kernel.mojo:26-314) and the Python
// post-processing of _CausalConv1dFn.backward
// (src/causal_conv1d_mojo/_fn.py:274-332).
//
// dweight/dbias are reduced deterministically: each block writes its
// partial sums (per channel, W+1 floats) into a workspace slot, and
// finalize_kernel adds the slots in a fixed order, writing fp32
// [dweight | dbias] plus optional dtype copies.  No atomics, no zeroing.
//
//  * bwd_seq_kernel  - unit-stride seqlen.  A warp walks a segment of one
//    (b, c) row from its last chunk to its first; dpre of the chunk to the
//    right is carried in registers, so dx needs no recomputation of the
//    right halo except once per segment.  The next chunk to the left is
//    prefetched while the current one is computed.
//  * bwd_chan_kernel - unit-stride dim (channel-last).  A lane owns VC
//    channels and walks time forwards; dx[p] is emitted W-1 steps after p,
//    once dpre[p .. p+W-1] are known.  The warps of a block share one
//    channel group and their partials are summed in shared memory.
#include "cc1d_dispatch.cuh"

namespace cc1d {

namespace {

constexpr int kThreads = 256;

template <typename T, int W, bool VEC, bool HAS_SEQ>
__global__ void __launch_bounds__(kThreads) bwd_seq_kernel(const BwdArgs a) {
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int CH = 32 * V;
  constexpr int H = W - 1;
  static_assert(H >= 1 && H <= V, "halo must fit in one lane vector");
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const T* __restrict__ dfin = static_cast<const T*>(a.dfin);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ dx = static_cast<T*>(a.dx);
  T* __restrict__ dinit = static_cast<T*>(a.dinit);
  const int lane = threadIdx.x & 31;
  const i64 nwarps = ((i64)gridDim.x * blockDim.x) >> 5;
  const int silu = a.silu;

  for (i64 item = ((i64)blockIdx.x * blockDim.x + threadIdx.x) >> 5; item < a.n_items; item += nwarps) {
    const i64 row = item / a.nseg;
    const i64 seg = item - row * a.nseg;
    const i64 b = row / a.D;
    const i64 c = row - b * a.D;
    float wv[W];
#pragma unroll
    for (int k = 0; k < W; ++k) wv[k] = Cvt<T>::f(wt[c * a.ws_c + k * a.ws_k]);
    const float bv = bias ? Cvt<T>::f(bias[c * a.bs]) : 0.f;
    const T* __restrict__ xr = x + b * a.xs_b + c * a.xs_c;
    const T* __restrict__ gr = dout + b * a.gs_b + c * a.gs_c;
    T* __restrict__ dxr = dx + b * a.dxs_b + c * a.dxs_c;
    const int* __restrict__ sr = HAS_SEQ ? seq + b * a.ss_b : nullptr;
    const T* __restrict__ ir = init ? init + b * a.is_b + c * a.is_c : nullptr;
    const T* __restrict__ fr = dfin ? dfin + b * a.fs_b + c * a.fs_c : nullptr;
    const i64 t_beg = seg * a.seg_len;
    const i64 t_end = min(a.L, t_beg + a.seg_len);

    // dpre (and seq ids) of the H positions right after the segment.
    float cd[H];
    int cs[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const i64 pos = t_end + j;
      cd[j] = 0.f;
      cs[j] = kNoSeq;
      if (pos < a.L) {
        const int cur = HAS_SEQ ? sr[pos * a.ss_l] : 0;
        float pre = bv;
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const i64 q = pos - H + k;
          float val = 0.f;
          int sq = kNoSeq;
          if (q >= 0) {
            val = Cvt<T>::f(xr[q * a.xs_l]);
            if (HAS_SEQ) sq = sr[q * a.ss_l];
          } else if (ir) {
            val = Cvt<T>::f(ir[(q + H) * a.is_l]);
          }
          if (!HAS_SEQ || sq == cur) pre = fmaf(wv[k], val, pre);
        }
        float g = Cvt<T>::f(gr[pos * a.gs_l]);
        if (silu) g *= silu_grad_f(pre);
        if (HAS_SEQ && cur < 0) g = 0.f;
        cd[j] = g;
        cs[j] = cur;
      }
    }

    float dwl[W];
#pragma unroll
    for (int k = 0; k < W; ++k) dwl[k] = 0.f;
    float dbl = 0.f;

    const i64 nch = ceil_div(t_end - t_beg, (i64)CH);
    // Current chunk registers (prefetched one chunk ahead).
    float xc[V], gc[V];
    int sc[V];
    int nvc;
    {
      const i64 t = t_beg + (nch - 1) * CH + lane * V;
      const i64 rem = t_end - t;
      nvc = rem >= V ? V : (rem > 0 ? (int)rem : 0);
      load_strided<T, V, VEC>(xr + t * a.xs_l, a.xs_l, nvc, xc);
      load_strided<T, V, VEC>(gr + t * a.gs_l, a.gs_l, nvc, gc);
      if (HAS_SEQ) {
#pragma unroll
        for (int i = 0; i < V; ++i) sc[i] = (i < nvc) ? sr[(t + i) * a.ss_l] : kNoSeq;
      }
    }
    for (i64 ci = nch - 1; ci >= 0; --ci) {
      const i64 t0 = t_beg + ci * CH;
      const i64 t = t0 + lane * V;
      // Prefetch the chunk to the left (always full: only the last chunk of
      // a segment can be partial).
      float xn[V], gn[V];
      int sn[V];
      if (ci > 0) {
        const i64 tn = t - CH;
        load_strided<T, V, VEC>(xr + tn * a.xs_l, a.xs_l, V, xn);
        load_strided<T, V, VEC>(gr + tn * a.gs_l, a.gs_l, V, gn);
        if (HAS_SEQ) {
#pragma unroll
          for (int i = 0; i < V; ++i) sn[i] = sr[(tn + i) * a.ss_l];
        }
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          xn[i] = 0.f;
          gn[i] = 0.f;
          sn[i] = kNoSeq;
        }
      }
      // Left halo (x and seq ids at t-H .. t-1).
      float h[H];
      int hs[H];
#pragma unroll
      for (int j = 0; j < H; ++j) {
        h[j] = __shfl_up_sync(kFull, xc[V - H + j], 1);
        hs[j] = HAS_SEQ ? __shfl_up_sync(kFull, sc[V - H + j], 1) : 0;
        const float h31 = __shfl_sync(kFull, xn[V - H + j], 31);
        const int s31 = HAS_SEQ ? __shfl_sync(kFull, sn[V - H + j], 31) : 0;
        if (lane == 0) {
          if (ci > 0) {
            h[j] = h31;
            hs[j] = s31;
          } else {
            const i64 p = t0 - H + j;
            h[j] = 0.f;
            hs[j] = kNoSeq;
            if (p >= 0) {
              h[j] = Cvt<T>::f(xr[p * a.xs_l]);
              if (HAS_SEQ) hs[j] = sr[p * a.ss_l];
            } else if (ir) {
              h[j] = Cvt<T>::f(ir[(p + H) * a.is_l]);
            }
          }
        }
      }
      // dpre of the lane's V positions.
      float dp[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int cur = HAS_SEQ ? sc[i] : 0;
        float pre = bv;
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const int q = i - H + k;
          const float val = q >= 0 ? xc[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H];
          if (HAS_SEQ) {
            const int sq = q >= 0 ? sc[q >= 0 ? q : 0] : hs[q >= 0 ? 0 : q + H];
            if (sq == cur) pre = fmaf(wv[k], val, pre);
          } else {
            pre = fmaf(wv[k], val, pre);
          }
        }
        float g = gc[i];
        if (silu) g *= silu_grad_f(pre);
        if (HAS_SEQ && cur < 0) g = 0.f;
        if (i >= nvc) g = 0.f;
        dp[i] = g;
      }
      // Right halo of dpre (positions t+V .. t+V+H-1).
      float rd[H];
      int rs[H];
#pragma unroll
      for (int j = 0; j < H; ++j) {
        rd[j] = __shfl_down_sync(kFull, dp[j], 1);
        rs[j] = HAS_SEQ ? __shfl_down_sync(kFull, sc[j], 1) : 0;
        if (lane == 31) {
          rd[j] = cd[j];
          rs[j] = cs[j];
        }
      }
      // dx of the lane's positions.
      float o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int cur = HAS_SEQ ? sc[i] : 0;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int q = i + j;
          const float val = q < V ? dp[q < V ? q : 0] : rd[q < V ? 0 : q - V];
          if (HAS_SEQ) {
            const int sq = q < V ? sc[q < V ? q : 0] : rs[q < V ? 0 : q - V];
            if (sq == cur) acc = fmaf(wv[H - j], val, acc);
          } else {
            acc = fmaf(wv[H - j], val, acc);
          }
        }
        if (fr) {
          const i64 qf = t + i + H - a.L;
          if (qf >= 0 && i < nvc) acc += Cvt<T>::f(fr[qf * a.fs_l]);
        }
        o[i] = acc;
      }
      if (nvc > 0) store_strided<T, V, VEC>(dxr + t * a.dxs_l, a.dxs_l, nvc, o);
      // dweight / dbias partials.
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int cur = HAS_SEQ ? sc[i] : 0;
        dbl += dp[i];
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const int q = i - H + k;
          const float val = q >= 0 ? xc[q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H];
          if (HAS_SEQ) {
            const int sq = q >= 0 ? sc[q >= 0 ? q : 0] : hs[q >= 0 ? 0 : q + H];
            if (sq == cur) dwl[k] = fmaf(dp[i], val, dwl[k]);
          } else {
            dwl[k] = fmaf(dp[i], val, dwl[k]);
          }
        }
      }
      // dinitial_states (lane 0 of the chunk holding t = 0).
      if (t0 == 0 && lane == 0 && dinit != nullptr) {
#pragma unroll
        for (int i = 0; i < H; ++i) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k <= i; ++k) acc = fmaf(wv[k], dp[i - k], acc);
          if (fr && i - a.L >= 0) acc += Cvt<T>::f(fr[(i - a.L) * a.fs_l]);
          dinit[b * a.dis_b + c * a.dis_c + i * a.dis_l] = Cvt<T>::to(acc);
        }
      }
      // Carry this chunk's first H dpre values to the chunk on the left.
#pragma unroll
      for (int j = 0; j < H; ++j) {
        cd[j] = __shfl_sync(kFull, dp[j], 0);
        cs[j] = HAS_SEQ ? __shfl_sync(kFull, sc[j], 0) : 0;
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        xc[i] = xn[i];
        gc[i] = gn[i];
        sc[i] = sn[i];
      }
      nvc = V;
    }

    // Warp-reduce the partial sums; lane 0 writes this item's slot.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
      for (int k = 0; k < W; ++k) dwl[k] += __shfl_xor_sync(kFull, dwl[k], off);
      dbl += __shfl_xor_sync(kFull, dbl, off);
    }
    if (lane == 0) {
      const i64 slot = b * a.nseg + seg;
      float* p = a.partials + (slot * a.D + c) * (W + 1);
#pragma unroll
      for (int k = 0; k < W; ++k) p[k] = dwl[k];
      p[W] = dbl;
    }
  }
}

template <typename T, int W, int VC, bool VEC, bool HAS_SEQ, int U>
__global__ void __launch_bounds__(kThreads) bwd_chan_kernel(const BwdArgs a) {
  constexpr int H = W - 1;
  constexpr int E = VC * (W + 1);
  extern __shared__ float red[];  // [warps][E][32]
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ dout = static_cast<const T*>(a.dout);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const T* __restrict__ dfin = static_cast<const T*>(a.dfin);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ dx = static_cast<T*>(a.dx);
  T* __restrict__ dinit = static_cast<T*>(a.dinit);
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int silu = a.silu;
  const i64 grp = blockIdx.x / a.splits;
  const i64 split = blockIdx.x - grp * a.splits;
  const i64 c0 = (grp * 32 + lane) * VC;
  const i64 ncl = a.D - c0;
  const int nc = ncl >= VC ? VC : (ncl > 0 ? (int)ncl : 0);
  const i64 R = a.B * a.L;
  const i64 cr0 = split * a.rows_per_split;
  const i64 cr1 = min(R, cr0 + a.rows_per_split);
  const i64 per = ceil_div(cr1 - cr0, wpb);
  i64 r = cr0 + wib * per;
  const i64 r_end = min(cr1, r + per);

  float wv[VC][W], bv[VC];
  float dwa[VC][W], dba[VC];
#pragma unroll
  for (int v = 0; v < VC; ++v) {
#pragma unroll
    for (int k = 0; k < W; ++k) {
      wv[v][k] = v < nc ? Cvt<T>::f(wt[(c0 + v) * a.ws_c + k * a.ws_k]) : 0.f;
      dwa[v][k] = 0.f;
    }
    bv[v] = (bias && v < nc) ? Cvt<T>::f(bias[(c0 + v) * a.bs]) : 0.f;
    dba[v] = 0.f;
  }

  if (nc > 0) {
    while (r < r_end) {
      const i64 b = r / a.L;
      const i64 t_start = r - b * a.L;
      const i64 t_stop = min(a.L, t_start + (r_end - r));
      r += t_stop - t_start;
      const T* __restrict__ xb = x + b * a.xs_b + c0 * a.xs_c;
      const T* __restrict__ gb = dout + b * a.gs_b + c0 * a.gs_c;
      T* __restrict__ dxb = dx + b * a.dxs_b + c0 * a.dxs_c;
      const int* __restrict__ sb = HAS_SEQ ? seq + b * a.ss_b : nullptr;

      // Windows over positions t-H .. t-1: x (xc), dpre and seq ids.
      float xw[H][VC], pw[H][VC];
      int sw[H];
#pragma unroll
      for (int j = 0; j < H; ++j) {
        const i64 p = t_start - H + j;
        if (p >= 0) {
          load_strided<T, VC, VEC>(xb + p * a.xs_l, a.xs_c, nc, xw[j]);
          sw[j] = HAS_SEQ ? sb[p * a.ss_l] : 0;
        } else {
#pragma unroll
          for (int v = 0; v < VC; ++v)
            xw[j][v] = (init && v < nc) ? Cvt<T>::f(init[b * a.is_b + (c0 + v) * a.is_c + (p + H) * a.is_l]) : 0.f;
          sw[j] = kNoSeq;
        }
#pragma unroll
        for (int v = 0; v < VC; ++v) pw[j][v] = 0.f;
      }

      const i64 t_last = t_stop + H;  // dx[p] is emitted at step p + H
      i64 t = t_start;
      while (t < t_last) {
        const i64 left = t_last - t;
        const int nu = left >= U ? U : (int)left;
        float xv[U][VC], gv[U][VC];
        int sid[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const i64 tt = t + u;
          if (u < nu && tt < a.L) {
            load_strided<T, VC, VEC>(xb + tt * a.xs_l, a.xs_c, nc, xv[u]);
            load_strided<T, VC, VEC>(gb + tt * a.gs_l, a.gs_c, nc, gv[u]);
            sid[u] = HAS_SEQ ? sb[tt * a.ss_l] : 0;
          } else {
#pragma unroll
            for (int v = 0; v < VC; ++v) {
              xv[u][v] = 0.f;
              gv[u][v] = 0.f;
            }
            sid[u] = kNoSeq;
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (u < nu) {
            const i64 tt = t + u;
            float dp[VC];
#pragma unroll
            for (int v = 0; v < VC; ++v) {
              float pre = bv[v];
#pragma unroll
              for (int k = 0; k < H; ++k)
                if (!HAS_SEQ || sw[k] == sid[u]) pre = fmaf(wv[v][k], xw[k][v], pre);
              pre = fmaf(wv[v][H], xv[u][v], pre);
              float g = gv[u][v];
              if (silu) g *= silu_grad_f(pre);
              if (HAS_SEQ && sid[u] < 0) g = 0.f;
              dp[v] = g;
            }
            if (tt < t_stop) {
#pragma unroll
              for (int v = 0; v < VC; ++v) {
                dba[v] += dp[v];
#pragma unroll
                for (int k = 0; k < H; ++k)
                  if (!HAS_SEQ || sw[k] == sid[u]) dwa[v][k] = fmaf(dp[v], xw[k][v], dwa[v][k]);
                dwa[v][H] = fmaf(dp[v], xv[u][v], dwa[v][H]);
              }
            }
            const i64 p = tt - H;
            // dinit (p < 0) is emitted only by the run that starts at t = 0:
            // a run starting later has no dpre for positions before it.
            if (p >= t_start || (t_start == 0 && p < 0 && dinit != nullptr)) {
              const int sp = sw[0];
              float o[VC];
#pragma unroll
              for (int v = 0; v < VC; ++v) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < H; ++j)
                  if (!HAS_SEQ || sw[j] == sp) acc = fmaf(wv[v][H - j], pw[j][v], acc);
                if (!HAS_SEQ || sid[u] == sp) acc = fmaf(wv[v][0], dp[v], acc);
                o[v] = acc;
              }
              if (dfin) {
                const i64 qf = p + H - a.L;
                if (qf >= 0) {
#pragma unroll
                  for (int v = 0; v < VC; ++v)
                    if (v < nc) o[v] += Cvt<T>::f(dfin[b * a.fs_b + (c0 + v) * a.fs_c + qf * a.fs_l]);
                }
              }
              if (p >= 0) {
                store_strided<T, VC, VEC>(dxb + p * a.dxs_l, a.dxs_c, nc, o);
              } else {
#pragma unroll
                for (int v = 0; v < VC; ++v)
                  if (v < nc) dinit[b * a.dis_b + (c0 + v) * a.dis_c + (p + H) * a.dis_l] = Cvt<T>::to(o[v]);
              }
            }
#pragma unroll
            for (int j = 0; j < H - 1; ++j) {
#pragma unroll
              for (int v = 0; v < VC; ++v) {
                xw[j][v] = xw[j + 1][v];
                pw[j][v] = pw[j + 1][v];
              }
              sw[j] = sw[j + 1];
            }
#pragma unroll
            for (int v = 0; v < VC; ++v) {
              xw[H - 1][v] = xv[u][v];
              pw[H - 1][v] = dp[v];
            }
            sw[H - 1] = sid[u];
          }
        }
        t += nu;
      }
    }
  }

  // Sum the warps' partials of this block's channel group in shared memory.
#pragma unroll
  for (int v = 0; v < VC; ++v) {
#pragma unroll
    for (int k = 0; k < W; ++k) red[(wib * E + v * (W + 1) + k) * 32 + lane] = dwa[v][k];
    red[(wib * E + v * (W + 1) + W) * 32 + lane] = dba[v];
  }
  __syncthreads();
  if (wib == 0 && nc > 0) {
    float* p = a.partials + (split * a.D + c0) * (W + 1);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float s = 0.f;
      for (int w2 = 0; w2 < wpb; ++w2) s += red[(w2 * E + e) * 32 + lane];
      if (e < nc * (W + 1)) p[e] = s;
    }
  }
}

// Sums the partial slots: a block owns 32 consecutive outputs (one per lane,
// so every load is a coalesced 128-byte row segment); warp w adds slots
// w, w+8, w+16, ... in order, then warp 0 adds the 8 warp sums in order.
// The summation order depends only on the slot count, so results are
// reproducible run to run.  Writes dwdb[c*W+k] (dweight) and dwdb[D*W+c]
// (dbias), plus optional dtype copies.
constexpr int kFinWarps = 8;

template <typename T, int W>
__global__ void __launch_bounds__(kFinWarps * 32) finalize_kernel(const FinalizeArgs a) {
  __shared__ float part[kFinWarps][32];
  griddep_wait();  // the partials come from the backward kernel just before
  griddep_launch_dependents();
  const i64 n = a.D * (W + 1);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const i64 e = (i64)blockIdx.x * 32 + lane;
  float s = 0.f;
  if (e < n)
    for (i64 i = warp; i < a.n_partials; i += kFinWarps) s += a.partials[i * n + e];
  part[warp][lane] = s;
  __syncthreads();
  if (warp != 0 || e >= n) return;
  s = part[0][lane];
#pragma unroll
  for (int w2 = 1; w2 < kFinWarps; ++w2) s += part[w2][lane];
  const i64 c = e / (W + 1);
  const int k = (int)(e - c * (W + 1));
  if (k < W) {
    a.dwdb[c * W + k] = s;
    if (a.dw_out) static_cast<T*>(a.dw_out)[c * a.dws_c + k * a.dws_k] = Cvt<T>::to(s);
  } else {
    if (!a.has_bias) s = 0.f;
    a.dwdb[a.D * W + c] = s;
    if (a.db_out && a.has_bias) static_cast<T*>(a.db_out)[c * a.dbs] = Cvt<T>::to(s);
  }
}

// seqlen == 0: dinitial_states = dfinal_states (or zeros).
template <typename T, int W>
__global__ void bwd_empty_kernel(const BwdArgs a) {
  constexpr int H = W - 1;
  const i64 n = a.B * a.D * H;
  for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (i64)gridDim.x * blockDim.x) {
    const i64 j = e % H;
    const i64 bc = e / H;
    const i64 c = bc % a.D;
    const i64 b = bc / a.D;
    const T* dfin = static_cast<const T*>(a.dfin);
    T v = dfin ? dfin[b * a.fs_b + c * a.fs_c + j * a.fs_l] : Cvt<T>::to(0.f);
    static_cast<T*>(a.dinit)[b * a.dis_b + c * a.dis_c + j * a.dis_l] = v;
  }
}

template <typename T>
constexpr int chan_vc() {
  return sizeof(T) == 4 ? 1 : 2;
}
constexpr int kChanUnroll = 4;

template <typename T>
bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0;
}

template <typename T, int W>
size_t chan_smem() {
  return (size_t)(kThreads / 32) * chan_vc<T>() * (W + 1) * 32 * sizeof(float);
}

struct PlanBwd {
  const BwdArgs& a;
  Plan* plan;
  template <typename T, int W>
  cudaError_t operator()() {
    DeviceInfo dev;
    cudaError_t e = device_info(&dev);
    if (e != cudaSuccess) return e;
    constexpr int V = 16 / (int)sizeof(T);
    constexpr int VC = chan_vc<T>();
    const bool seq_unit = (a.L == 1) || (a.xs_l == 1 && a.gs_l == 1 && a.dxs_l == 1);
    const bool chan_unit = (a.D == 1) || (a.xs_c == 1 && a.gs_c == 1 && a.dxs_c == 1);
    Layout layout;
    if (seq_unit && chan_unit)
      layout = (a.L >= a.D) ? kSeq : kChan;
    else if (seq_unit)
      layout = kSeq;
    else if (chan_unit)
      layout = kChan;
    else
      layout = kSeq;
    plan->layout = layout;
    plan->threads = kThreads;
    const int wpb = kThreads / 32;
    if (layout == kSeq) {
      const bool vec = a.xs_l == 1 && a.gs_l == 1 && a.dxs_l == 1 && aligned<T>(a.x, 16) &&
                       aligned<T>(a.dout, 16) && aligned<T>(a.dx, 16) &&
                       (a.B == 1 || (a.xs_b % V == 0 && a.gs_b % V == 0 && a.dxs_b % V == 0)) &&
                       (a.D == 1 || (a.xs_c % V == 0 && a.gs_c % V == 0 && a.dxs_c % V == 0));
      plan->vec = vec;
      int nb = 1;
      static std::atomic<int> occ{0};
      e = blocks_per_sm(bwd_seq_kernel<T, W, true, false>, kThreads, 0, occ, &nb);
      if (e != cudaSuccess) return e;
      const i64 resident_warps = (i64)dev.sms * nb * wpb;
      const i64 rows = a.B * a.D;
      const i64 chunk = 32 * V;
      i64 nseg = 1;
      if (rows < 4 * resident_warps) nseg = ceil_div(4 * resident_warps, rows);
      nseg = std::min<i64>(nseg, ceil_div(a.L, chunk));
      if (nseg < 1) nseg = 1;
      const i64 seg_len = ceil_div(ceil_div(a.L, nseg), chunk) * chunk;
      nseg = ceil_div(a.L, seg_len);
      plan->nseg = nseg;
      plan->seg_len = seg_len;
      plan->n_items = rows * nseg;
      plan->grid = std::min<i64>(ceil_div(plan->n_items, wpb), (i64)dev.sms * nb);
      plan->n_partials = a.B * nseg;
    } else {
      const int vb = VC * (int)sizeof(T);
      const bool vec = a.xs_c == 1 && a.gs_c == 1 && a.dxs_c == 1 && aligned<T>(a.x, vb) &&
                       aligned<T>(a.dout, vb) && aligned<T>(a.dx, vb) &&
                       (a.B == 1 || (a.xs_b % VC == 0 && a.gs_b % VC == 0 && a.dxs_b % VC == 0)) &&
                       (a.L == 1 || (a.xs_l % VC == 0 && a.gs_l % VC == 0 && a.dxs_l % VC == 0));
      plan->vec = vec;
      int nb = 1;
      static std::atomic<int> occ{0};
      e = blocks_per_sm(bwd_chan_kernel<T, W, VC, true, false, kChanUnroll>, kThreads, chan_smem<T, W>(), occ,
                        &nb);
      if (e != cudaSuccess) return e;
      const i64 groups = ceil_div(a.D, 32 * VC);
      const i64 R = a.B * a.L;
      const i64 target = (i64)dev.sms * nb;
      i64 splits = std::max<i64>(1, target / groups);
      i64 rps = ceil_div(R, splits);
      rps = std::max<i64>(rps, (i64)wpb * 16);
      splits = ceil_div(R, rps);
      plan->groups = groups;
      plan->splits = splits;
      plan->rows_per_split = rps;
      plan->grid = groups * splits;
      plan->n_partials = splits;
    }
    if (a.B * a.D * a.L == 0) {
      plan->grid = 0;
      plan->n_partials = 0;
    }
    return cudaSuccess;
  }
};

struct LaunchBwd {
  BwdArgs a;
  const Plan& plan;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    constexpr int VC = chan_vc<T>();
    a.nseg = plan.nseg;
    a.seg_len = plan.seg_len;
    a.n_items = plan.n_items;
    a.splits = plan.splits;
    a.rows_per_split = plan.rows_per_split;
    const dim3 grid((unsigned)plan.grid), block(plan.threads);
    const bool hs = a.seq != nullptr;
    if (plan.layout == kSeq) {
      if (plan.vec) {
        if (hs) bwd_seq_kernel<T, W, true, true><<<grid, block, 0, stream>>>(a);
        else bwd_seq_kernel<T, W, true, false><<<grid, block, 0, stream>>>(a);
      } else {
        if (hs) bwd_seq_kernel<T, W, false, true><<<grid, block, 0, stream>>>(a);
        else bwd_seq_kernel<T, W, false, false><<<grid, block, 0, stream>>>(a);
      }
    } else {
      const size_t smem = chan_smem<T, W>();
      if (plan.vec) {
        if (hs) bwd_chan_kernel<T, W, VC, true, true, kChanUnroll><<<grid, block, smem, stream>>>(a);
        else bwd_chan_kernel<T, W, VC, true, false, kChanUnroll><<<grid, block, smem, stream>>>(a);
      } else {
        if (hs) bwd_chan_kernel<T, W, VC, false, true, kChanUnroll><<<grid, block, smem, stream>>>(a);
        else bwd_chan_kernel<T, W, VC, false, false, kChanUnroll><<<grid, block, smem, stream>>>(a);
      }
    }
    return cudaGetLastError();
  }
};

struct LaunchFinalize {
  const FinalizeArgs& a;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    const i64 n = a.D * (W + 1);
    if (n == 0) return cudaSuccess;
    return launch_pdl(finalize_kernel<T, W>, dim3((unsigned)ceil_div(n, (i64)32)), dim3(kFinWarps * 32), 0, stream, a);
  }
};

struct LaunchBwdEmpty {
  const BwdArgs& a;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    const i64 n = a.B * a.D * (W - 1);
    if (n == 0 || a.dinit == nullptr) return cudaSuccess;
    const int threads = 256;
    const i64 blocks = std::min<i64>(ceil_div(n, threads), 4096);
    bwd_empty_kernel<T, W><<<(unsigned)blocks, threads, 0, stream>>>(a);
    return cudaGetLastError();
  }
};

}  // namespace

cudaError_t plan_bwd(int dtype, int width, const BwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, PlanBwd{a, plan});
}

cudaError_t launch_bwd(int dtype, int width, BwdArgs a, const Plan& plan, cudaStream_t stream) {
  if (plan.grid <= 0) return cudaSuccess;
  return dispatch(dtype, width, LaunchBwd{a, plan, stream});
}

cudaError_t launch_finalize(int dtype, int width, const FinalizeArgs& a, cudaStream_t stream) {
  return dispatch(dtype, width, LaunchFinalize{a, stream});
}

cudaError_t launch_bwd_empty_seq(int dtype, int width, const BwdArgs& a, cudaStream_t stream) {
  return dispatch(dtype, width, LaunchBwdEmpty{a, stream});
}

}  // namespace cc1d
