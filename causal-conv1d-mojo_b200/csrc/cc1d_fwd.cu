// Forward kernels of causal_conv1d_fn for sm_100a.
//
//   out[b,c,t] = act(bias[c] + sum_k w[c,k] * xc[b,c,t-(W-1)+k])
//
// xc is x preceded by initial_states (or zeros).  With seq_idx a tap is
// used only when seq_idx[b,src] == seq_idx[b,t], and seq_idx[b,t] < 0
// forces out = 0.  final_states = last W-1 columns of xc, copied exactly.
// Semantics follow the reference CPU kernel
// (src/causal_conv1d_mojo/fwd_cpu/kernel.mojo:64-117) and the pure-PyTorch
// reference (src/causal_conv1d_mojo/reference.py:21-59, final_states from
// cat([initial_states, x]) as at reference.py:50-56).
//
// Two layouts (chosen by the ABI layer from the strides):
//  * fwd_seq_kernel  - seqlen is the unit-stride axis.  A warp walks a
//    segment of one (b, c) row in chunks of 32 lanes x 16 bytes; the W-1
//    element halo of lane i comes from lane i-1 by shuffle (lane 0 takes it
//    from the previous chunk of the same pass, or reads it once per pass).
//  * fwd_chan_kernel - dim is the unit-stride axis (channel-last, the Mamba
//    layout).  A lane owns VC adjacent channels and walks a contiguous run of
//    (b, t) rows keeping the last W-1 rows in registers, so every x element
//    is loaded once apart from a W-1 row halo per run.
// Both read x exactly once from HBM and write out once: the kernels are
// bound by HBM bandwidth (about 4 bytes per element for 16-bit types).
#include "cc1d_dispatch.cuh"

namespace cc1d {

namespace {

constexpr int kThreads = 256;

template <typename T, int W, bool VEC, bool HAS_SEQ, int U>
__global__ void __launch_bounds__(kThreads) fwd_seq_kernel(const FwdArgs a) {
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int CH = 32 * V;
  constexpr int H = W - 1;
  static_assert(H >= 1 && H <= V, "halo must fit in one lane vector");
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ out = static_cast<T*>(a.out);
  T* __restrict__ fin = static_cast<T*>(a.fin);
  const int lane = threadIdx.x & 31;
  const i64 nwarps = ((i64)gridDim.x * blockDim.x) >> 5;

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
    T* __restrict__ orow = out + b * a.os_b + c * a.os_c;
    const int* __restrict__ sr = HAS_SEQ ? seq + b * a.ss_b : nullptr;
    const T* __restrict__ ir = init ? init + b * a.is_b + c * a.is_c : nullptr;
    const i64 t_beg = seg * a.seg_len;
    const i64 t_end = min(a.L, t_beg + a.seg_len);

    for (i64 t0 = t_beg; t0 < t_end; t0 += (i64)U * CH) {
      float xv[U][V];
      int sv[U][V];
      int nv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const i64 t = t0 + u * CH + lane * V;
        const i64 rem = t_end - t;
        nv[u] = rem >= V ? V : (rem > 0 ? (int)rem : 0);
        load_strided<T, V, VEC>(xr + t * a.xs_l, a.xs_l, nv[u], xv[u]);
        if (HAS_SEQ) {
#pragma unroll
          for (int i = 0; i < V; ++i) sv[u][i] = (i < nv[u]) ? sr[(t + i) * a.ss_l] : kNoSeq;
        }
      }
      // Halo of lane 0 in the first chunk of this pass.
      float h0[H];
      int hs0[H];
#pragma unroll
      for (int j = 0; j < H; ++j) {
        h0[j] = 0.f;
        hs0[j] = kNoSeq;
      }
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const i64 p = t0 - H + j;
          if (p >= 0) {
            h0[j] = Cvt<T>::f(xr[p * a.xs_l]);
            if (HAS_SEQ) hs0[j] = sr[p * a.ss_l];
          } else if (ir) {
            h0[j] = Cvt<T>::f(ir[(p + H) * a.is_l]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float h[H];
        int hs[H];
#pragma unroll
        for (int j = 0; j < H; ++j) {
          h[j] = __shfl_up_sync(kFull, xv[u][V - H + j], 1);
          hs[j] = HAS_SEQ ? __shfl_up_sync(kFull, sv[u][V - H + j], 1) : 0;
          if (u > 0) {
            const float hp = __shfl_sync(kFull, xv[u > 0 ? u - 1 : 0][V - H + j], 31);
            const int sp = HAS_SEQ ? __shfl_sync(kFull, sv[u > 0 ? u - 1 : 0][V - H + j], 31) : 0;
            if (lane == 0) {
              h[j] = hp;
              hs[j] = sp;
            }
          } else if (lane == 0) {
            h[j] = h0[j];
            hs[j] = hs0[j];
          }
        }
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int cur = HAS_SEQ ? sv[u][i] : 0;
          float acc = bv;
#pragma unroll
          for (int k = 0; k < W; ++k) {
            const int q = i - H + k;
            const float val = q >= 0 ? xv[u][q >= 0 ? q : 0] : h[q >= 0 ? 0 : q + H];
            if (HAS_SEQ) {
              const int sq = q >= 0 ? sv[u][q >= 0 ? q : 0] : hs[q >= 0 ? 0 : q + H];
              if (sq == cur) acc = fmaf(wv[k], val, acc);
            } else {
              acc = fmaf(wv[k], val, acc);
            }
          }
          if (a.silu) acc = silu_f(acc);
          if (HAS_SEQ && cur < 0) acc = 0.f;
          o[i] = acc;
        }
        const i64 t = t0 + u * CH + lane * V;
        if (nv[u] > 0) store_strided<T, V, VEC>(orow + t * a.os_l, a.os_l, nv[u], o);
      }
    }

    if (fin != nullptr && t_end == a.L && lane < H) {
      const i64 p = a.L - H + lane;
      T v = Cvt<T>::to(0.f);
      if (p >= 0)
        v = xr[p * a.xs_l];
      else if (ir)
        v = ir[(p + H) * a.is_l];
      fin[b * a.fs_b + c * a.fs_c + lane * a.fs_l] = v;
    }
  }
}

template <typename T, int W, int VC, bool VEC, bool HAS_SEQ, int U>
__global__ void __launch_bounds__(kThreads) fwd_chan_kernel(const FwdArgs a) {
  constexpr int H = W - 1;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ init = static_cast<const T*>(a.init);
  const int* __restrict__ seq = a.seq;
  T* __restrict__ out = static_cast<T*>(a.out);
  T* __restrict__ fin = static_cast<T*>(a.fin);
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const i64 grp = blockIdx.x / a.splits;
  const i64 split = blockIdx.x - grp * a.splits;
  const i64 c0 = (grp * 32 + lane) * VC;
  const i64 ncl = a.D - c0;
  const int nc = ncl >= VC ? VC : (ncl > 0 ? (int)ncl : 0);
  if (nc == 0) return;
  const i64 R = a.B * a.L;
  const i64 cr0 = split * a.rows_per_split;
  const i64 cr1 = min(R, cr0 + a.rows_per_split);
  const i64 per = ceil_div(cr1 - cr0, wpb);
  i64 r = cr0 + wib * per;
  const i64 r_end = min(cr1, r + per);

  float wv[VC][W], bv[VC];
#pragma unroll
  for (int v = 0; v < VC; ++v) {
#pragma unroll
    for (int k = 0; k < W; ++k) wv[v][k] = v < nc ? Cvt<T>::f(wt[(c0 + v) * a.ws_c + k * a.ws_k]) : 0.f;
    bv[v] = (bias && v < nc) ? Cvt<T>::f(bias[(c0 + v) * a.bs]) : 0.f;
  }

  while (r < r_end) {
    const i64 b = r / a.L;
    i64 t = r - b * a.L;
    const i64 t_stop = min(a.L, t + (r_end - r));
    r += t_stop - t;
    const T* __restrict__ xb = x + b * a.xs_b + c0 * a.xs_c;
    T* __restrict__ ob = out + b * a.os_b + c0 * a.os_c;
    const int* __restrict__ sb = HAS_SEQ ? seq + b * a.ss_b : nullptr;

    // Window of the H rows before t (initial_states / zeros before 0).
    float win[H][VC];
    int wsid[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const i64 p = t - H + j;
      if (p >= 0) {
        load_strided<T, VC, VEC>(xb + p * a.xs_l, a.xs_c, nc, win[j]);
        wsid[j] = HAS_SEQ ? sb[p * a.ss_l] : 0;
      } else {
#pragma unroll
        for (int v = 0; v < VC; ++v)
          win[j][v] = (init && v < nc) ? Cvt<T>::f(init[b * a.is_b + (c0 + v) * a.is_c + (p + H) * a.is_l]) : 0.f;
        wsid[j] = kNoSeq;
      }
    }

    while (t < t_stop) {
      const i64 left = t_stop - t;
      const int nu = left >= U ? U : (int)left;
      float xv[U][VC];
      int sid[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < nu) {
          load_strided<T, VC, VEC>(xb + (t + u) * a.xs_l, a.xs_c, nc, xv[u]);
          sid[u] = HAS_SEQ ? sb[(t + u) * a.ss_l] : 0;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (u < nu) {
          float o[VC];
#pragma unroll
          for (int v = 0; v < VC; ++v) {
            float acc = bv[v];
#pragma unroll
            for (int k = 0; k < H; ++k) {
              if (!HAS_SEQ || wsid[k] == sid[u]) acc = fmaf(wv[v][k], win[k][v], acc);
            }
            acc = fmaf(wv[v][H], xv[u][v], acc);
            if (a.silu) acc = silu_f(acc);
            if (HAS_SEQ && sid[u] < 0) acc = 0.f;
            o[v] = acc;
          }
          store_strided<T, VC, VEC>(ob + (t + u) * a.os_l, a.os_c, nc, o);
#pragma unroll
          for (int j = 0; j < H - 1; ++j) {
#pragma unroll
            for (int v = 0; v < VC; ++v) win[j][v] = win[j + 1][v];
            wsid[j] = wsid[j + 1];
          }
#pragma unroll
          for (int v = 0; v < VC; ++v) win[H - 1][v] = xv[u][v];
          wsid[H - 1] = sid[u];
        }
      }
      t += nu;
    }

    if (fin != nullptr && t_stop == a.L) {
#pragma unroll
      for (int j = 0; j < H; ++j)
#pragma unroll
        for (int v = 0; v < VC; ++v)
          if (v < nc) fin[b * a.fs_b + (c0 + v) * a.fs_c + j * a.fs_l] = Cvt<T>::to(win[j][v]);
    }
  }
}

// seqlen == 0: final_states = initial_states (or zeros).
template <typename T, int W>
__global__ void fwd_empty_kernel(const FwdArgs a) {
  constexpr int H = W - 1;
  const i64 n = a.B * a.D * H;
  for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (i64)gridDim.x * blockDim.x) {
    const i64 j = e % H;
    const i64 bc = e / H;
    const i64 c = bc % a.D;
    const i64 b = bc / a.D;
    const T* init = static_cast<const T*>(a.init);
    T v = init ? init[b * a.is_b + c * a.is_c + j * a.is_l] : Cvt<T>::to(0.f);
    static_cast<T*>(a.fin)[b * a.fs_b + c * a.fs_c + j * a.fs_l] = v;
  }
}

// Channels per lane of the channel-last kernel.
template <typename T>
constexpr int chan_vc() {
  return sizeof(T) == 4 ? 2 : 4;
}
constexpr int kSeqUnroll = 2;
constexpr int kChanUnroll = 4;

template <typename T>
bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0;
}

struct PlanFwd {
  const FwdArgs& a;
  Plan* plan;
  template <typename T, int W>
  cudaError_t operator()() {
    DeviceInfo dev;
    cudaError_t e = device_info(&dev);
    if (e != cudaSuccess) return e;
    constexpr int V = 16 / (int)sizeof(T);
    constexpr int VC = chan_vc<T>();
    const bool seq_unit = (a.L == 1) || (a.xs_l == 1 && a.os_l == 1);
    const bool chan_unit = (a.D == 1) || (a.xs_c == 1 && a.os_c == 1);
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
      const bool vec = a.xs_l == 1 && a.os_l == 1 && aligned<T>(a.x, 16) && aligned<T>(a.out, 16) &&
                       (a.B == 1 || (a.xs_b % V == 0 && a.os_b % V == 0)) &&
                       (a.D == 1 || (a.xs_c % V == 0 && a.os_c % V == 0));
      plan->vec = vec;
      int nb = 1;
      static std::atomic<int> occ{0};
      e = blocks_per_sm(fwd_seq_kernel<T, W, true, false, kSeqUnroll>, kThreads, 0, occ, &nb);
      if (e != cudaSuccess) return e;
      const i64 resident_warps = (i64)dev.sms * nb * wpb;
      const i64 rows = a.B * a.D;
      const i64 pass = (i64)kSeqUnroll * 32 * V;
      i64 nseg = 1;
      if (rows < 4 * resident_warps) nseg = ceil_div(4 * resident_warps, rows);
      nseg = std::min<i64>(nseg, ceil_div(a.L, pass));
      if (nseg < 1) nseg = 1;
      i64 seg_len = ceil_div(ceil_div(a.L, nseg), pass) * pass;
      nseg = ceil_div(a.L, seg_len);
      plan->nseg = nseg;
      plan->seg_len = seg_len;
      plan->n_items = rows * nseg;
      plan->grid = std::min<i64>(ceil_div(plan->n_items, wpb), (i64)dev.sms * nb);
    } else {
      const bool vec = a.xs_c == 1 && a.os_c == 1 && aligned<T>(a.x, VC * sizeof(T)) &&
                       aligned<T>(a.out, VC * sizeof(T)) && (a.B == 1 || (a.xs_b % VC == 0 && a.os_b % VC == 0)) &&
                       (a.L == 1 || (a.xs_l % VC == 0 && a.os_l % VC == 0));
      plan->vec = vec;
      int nb = 1;
      static std::atomic<int> occ{0};
      e = blocks_per_sm(fwd_chan_kernel<T, W, VC, true, false, kChanUnroll>, kThreads, 0, occ, &nb);
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
    }
    return cudaSuccess;
  }
};

struct LaunchFwd {
  FwdArgs a;
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
        if (hs) fwd_seq_kernel<T, W, true, true, kSeqUnroll><<<grid, block, 0, stream>>>(a);
        else fwd_seq_kernel<T, W, true, false, kSeqUnroll><<<grid, block, 0, stream>>>(a);
      } else {
        if (hs) fwd_seq_kernel<T, W, false, true, kSeqUnroll><<<grid, block, 0, stream>>>(a);
        else fwd_seq_kernel<T, W, false, false, kSeqUnroll><<<grid, block, 0, stream>>>(a);
      }
    } else {
      if (plan.vec) {
        if (hs) fwd_chan_kernel<T, W, VC, true, true, kChanUnroll><<<grid, block, 0, stream>>>(a);
        else fwd_chan_kernel<T, W, VC, true, false, kChanUnroll><<<grid, block, 0, stream>>>(a);
      } else {
        if (hs) fwd_chan_kernel<T, W, VC, false, true, kChanUnroll><<<grid, block, 0, stream>>>(a);
        else fwd_chan_kernel<T, W, VC, false, false, kChanUnroll><<<grid, block, 0, stream>>>(a);
      }
    }
    return cudaGetLastError();
  }
};

struct LaunchFwdEmpty {
  const FwdArgs& a;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    const i64 n = a.B * a.D * (W - 1);
    if (n == 0 || a.fin == nullptr) return cudaSuccess;
    const int threads = 256;
    const i64 blocks = std::min<i64>(ceil_div(n, threads), 4096);
    fwd_empty_kernel<T, W><<<(unsigned)blocks, threads, 0, stream>>>(a);
    return cudaGetLastError();
  }
};

}  // namespace

cudaError_t plan_fwd(int dtype, int width, const FwdArgs& a, Plan* plan) {
  return dispatch(dtype, width, PlanFwd{a, plan});
}

cudaError_t launch_fwd(int dtype, int width, FwdArgs a, const Plan& plan, cudaStream_t stream) {
  if (plan.grid <= 0) return cudaSuccess;
  return dispatch(dtype, width, LaunchFwd{a, plan, stream});
}

cudaError_t launch_fwd_empty_seq(int dtype, int width, const FwdArgs& a, cudaStream_t stream) {
  return dispatch(dtype, width, LaunchFwdEmpty{a, stream});
}

}  // namespace cc1d
