// Decode-step kernel of causal_conv1d_update and the varlen state gather
// of causal_conv1d_varlen_states, for sm_100a.
//
// update_kernel: one thread per (b, c).  Semantics follow the reference
// CPU kernel (src/causal_conv1d_mojo/update_cpu/kernel.mojo:52-139) and the
// pure-PyTorch reference (src/causal_conv1d_mojo/reference.py:62-121):
//   * conv_state_indices[b] < 0: out[b] = 0 and the state row is untouched;
//     otherwise row conv_state_indices[b] (or b) of conv_state serves b;
//   * linear mode: window = last W-1 state values, then the new state is
//     the last state_len values of cat([state, x]);
//   * circular mode: window = state[(cs-(W-1)+j) mod S], x written at
//     (cs+i) mod S, cs = cache_seqlens[b] (floor modulo S);
//   * out[i] = act(bias + sum_k w[k] * window[k]) with the same fp32 tap
//     order as the forward kernel, so decoding token by token reproduces the
//     forward pass bit for bit.
//
// The same semantics run in specialised kernels, chosen by the launcher
// from the layout (every one issues all its loads before any store):
//   update_vec_kernel      one token: linear with state_len W-1 (packed or
//                          channel-last pools) or circular channel-last
//                          states; 4 channels per thread, vectors
//   update_lin_kernel      linear, seqlen <= 8, state_len <= 16, any strides
//   update_circ_row_kernel one token, circular, 16- or 32-byte state rows
//   update_circ_kernel     one token, circular, any row size / strides
//   update_kernel          everything else
// Every kernel but update_circ_kernel / update_kernel is launched with
// programmatic dependent launch (waits on griddepcontrol before touching
// memory).
//
// varlen_states_kernel: one thread per (sequence, slot, channel) on a 3-D
// grid (channel blocks, slot, sequence), channel fastest, so reads of x rows
// and writes of the (batch, state_len, dim) output storage are both
// coalesced and no thread divides an index
// (src/causal_conv1d_mojo/causal_conv1d_varlen.py:29-61).
#include "cc1d_dispatch.cuh"

namespace cc1d {

namespace {

template <typename T, int W>
__global__ void __launch_bounds__(128) update_kernel(const UpdateArgs a) {
  constexpr int H = W - 1;
  const i64 cblocks = ceil_div(a.D, (i64)blockDim.x);
  const i64 b = blockIdx.x / cblocks;
  const i64 c = (blockIdx.x - b * cblocks) * blockDim.x + threadIdx.x;
  if (c >= a.D) return;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  T* __restrict__ out = static_cast<T*>(a.out);
  T* __restrict__ ob = out + b * a.os_b + c * a.os_c;
  i64 row = b;
  if (a.idx != nullptr) {
    const int r = a.idx[b];
    // Negative: padding token.  An index past the pool is invalid input; it
    // is treated like padding instead of touching memory outside conv_state.
    if (r < 0 || r >= a.state_rows) {
      for (i64 i = 0; i < a.L; ++i) ob[i * a.os_l] = Cvt<T>::to(0.f);
      return;
    }
    row = r;
  }
  T* __restrict__ st = static_cast<T*>(a.state) + row * a.ss_b + c * a.ss_c;
  const T* __restrict__ xb = x + b * a.xs_b + c * a.xs_c;
  float wv[W];
#pragma unroll
  for (int k = 0; k < W; ++k) wv[k] = Cvt<T>::f(wt[c * a.ws_c + k * a.ws_k]);
  const float bv = bias ? Cvt<T>::f(bias[c * a.bs]) : 0.f;
  const i64 S = a.S;
  float win[W];
  if (a.cache_seqlens != nullptr) {
    i64 cs = (i64)a.cache_seqlens[b] % S;
    if (cs < 0) cs += S;
    i64 ui = cs - H;
    if (ui < 0) ui += S;
#pragma unroll
    for (int j = 0; j < H; ++j) {
      win[j] = Cvt<T>::f(st[ui * a.ss_l]);
      ui = (ui + 1 == S) ? 0 : ui + 1;
    }
    for (i64 i = 0; i < a.L; ++i) {
      const T xv = xb[i * a.xs_l];
      st[ui * a.ss_l] = xv;
      ui = (ui + 1 == S) ? 0 : ui + 1;
      win[H] = Cvt<T>::f(xv);
      float acc = bv;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(wv[k], win[k], acc);
      if (a.silu) acc = silu_f(acc);
      ob[i * a.os_l] = Cvt<T>::to(acc);
#pragma unroll
      for (int k = 0; k < H; ++k) win[k] = win[k + 1];
    }
  } else {
    // History = the last H values of the old state.
#pragma unroll
    for (int j = 0; j < H; ++j) win[j] = Cvt<T>::f(st[(S - H + j) * a.ss_l]);
    // New state = last S values of cat([state, x]); ascending j only reads
    // positions that are not yet overwritten.
    for (i64 j = 0; j < S; ++j) {
      const i64 src = a.L + j;
      st[j * a.ss_l] = (src < S) ? st[src * a.ss_l] : xb[(src - S) * a.xs_l];
    }
    for (i64 i = 0; i < a.L; ++i) {
      win[H] = Cvt<T>::f(xb[i * a.xs_l]);
      float acc = bv;
#pragma unroll
      for (int k = 0; k < W; ++k) acc = fmaf(wv[k], win[k], acc);
      if (a.silu) acc = silu_f(acc);
      ob[i * a.os_l] = Cvt<T>::to(acc);
#pragma unroll
      for (int k = 0; k < H; ++k) win[k] = win[k + 1];
    }
  }
}

// Linear-mode decode step for short bursts (seqlen <= kLinLMax) and short
// states (state_len <= kLinSMax), any strides: one thread per (b, c); every
// load (the W-1 history, the whole old state row, the burst's x, weights,
// bias) is issued before any store, so a thread has one memory round trip
// after the pool index, and a warp's accesses cover 32 consecutive channels
// whatever the layout (packed rows, or channel-last state with unit channel
// stride).  Same tap order and SiLU as update_kernel.
constexpr int kLinLMax = 8;
constexpr int kLinSMax = 16;

// A 16-bit or 32-bit element, given its bits in the low bits of `h`.
template <typename T>
__device__ __forceinline__ float bits_to_float(uint32_t h);
template <>
__device__ __forceinline__ float bits_to_float<float>(uint32_t h) { return __uint_as_float(h); }
template <>
__device__ __forceinline__ float bits_to_float<__nv_bfloat16>(uint32_t h) { return __uint_as_float(h << 16); }
template <>
__device__ __forceinline__ float bits_to_float<__half>(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

// Raw bits of one element (state values are copied bit for bit).
template <typename T>
struct RawElem {
  typedef unsigned short type;
};
template <>
struct RawElem<float> {
  typedef unsigned int type;
};
template <typename T>
__device__ __forceinline__ float raw_to_float(typename RawElem<T>::type r) {
  return bits_to_float<T>((uint32_t)r);
}

// SFIX > 0: state_len == SFIX known at compile time (the serving layout
// state_len == W-1); 0: any state_len <= kLinSMax.  LFIX > 0: seqlen ==
// LFIX (no predicated-off token iterations are issued); 0: any seqlen <=
// kLinLMax.  Grid (channel blocks, batch).
template <typename T, int W, int SFIX, int LFIX>
__global__ void __launch_bounds__(128) update_lin_kernel(const UpdateArgs a) {
  griddep_wait();  // inputs and state may come from the previous kernel
  griddep_launch_dependents();
  typedef typename RawElem<T>::type R;
  constexpr int H = W - 1;
  constexpr int SM = SFIX > 0 ? SFIX : kLinSMax;
  const i64 b = blockIdx.y;
  const i64 c = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= a.D) return;
  constexpr int LM = LFIX > 0 ? LFIX : kLinLMax;
  const int L = LFIX > 0 ? LFIX : (int)a.L, S = SFIX > 0 ? SFIX : (int)a.S;
  T* __restrict__ ob = static_cast<T*>(a.out) + b * a.os_b + c * a.os_c;
  i64 row = b;
  if (a.idx != nullptr) {
    const int r = a.idx[b];
    if (r < 0 || r >= a.state_rows) {
#pragma unroll
      for (int i = 0; i < LM; ++i)
        if (i < L) ob[i * a.os_l] = Cvt<T>::to(0.f);
      return;
    }
    row = r;
  }
  R* __restrict__ st = reinterpret_cast<R*>(static_cast<T*>(a.state) + row * a.ss_b + c * a.ss_c);
  const R* __restrict__ xb = reinterpret_cast<const R*>(static_cast<const T*>(a.x) + b * a.xs_b + c * a.xs_c);
  // The state is held right-aligned in a shift register: reg[SM-S .. SM-1]
  // = old state; every register index below is a compile-time constant.
  R reg[SM], xv[LM];
#pragma unroll
  for (int q = 0; q < SM; ++q) {
    const int j = q - (SM - S);
    reg[q] = j >= 0 ? st[j * a.ss_l] : (R)0;
  }
#pragma unroll
  for (int i = 0; i < LM; ++i) xv[i] = i < L ? xb[i * a.xs_l] : (R)0;
  float wv[W];
#pragma unroll
  for (int k = 0; k < W; ++k) wv[k] = Cvt<T>::f(static_cast<const T*>(a.w)[c * a.ws_c + k * a.ws_k]);
  const float bv = a.bias ? Cvt<T>::f(static_cast<const T*>(a.bias)[c * a.bs]) : 0.f;
#pragma unroll
  for (int i = 0; i < LM; ++i) {
    if (i < L) {
      float acc = bv;
#pragma unroll
      for (int k = 0; k < H; ++k) acc = fmaf(wv[k], raw_to_float<T>(reg[SM - H + k]), acc);
      acc = fmaf(wv[H], raw_to_float<T>(xv[i]), acc);
      if (a.silu) acc = silu_f(acc);
      ob[i * a.os_l] = Cvt<T>::to(acc);
#pragma unroll
      for (int q = 0; q < SM - 1; ++q) reg[q] = reg[q + 1];
      reg[SM - 1] = xv[i];
    }
  }
  // New state = the last S values of cat([old, x]) = reg[SM-S .. SM-1].
#pragma unroll
  for (int q = 0; q < SM; ++q) {
    const int j = q - (SM - S);
    if (j >= 0) st[j * a.ss_l] = reg[q];
  }
}

// Largest vector (in elements, a power of two, at most 16 bytes) that
// divides a run of N contiguous elements of T.
template <typename T, int N>
constexpr int vec_elems() {
  int e = 16 / (int)sizeof(T);
  while (e > 1 && N % e != 0) e /= 2;
  return e;
}

// Plain (coherent) vector load, for data this kernel also writes.
template <typename T, int N>
__device__ __forceinline__ Pack<T, N> ld_pack_rw(const T* p) {
  Pack<T, N> pk;
  pk.raw = *reinterpret_cast<const typename Pack<T, N>::Raw*>(p);
  return pk;
}

// Channels per thread of the linear single-token update (B200, C3a shape:
// 4 -> 6.45 us, 8 -> 7.13 us, 2 -> 7.0 us).
#ifndef CC1D_VEC_V
#define CC1D_VEC_V 4
#endif
#ifndef CC1D_VEC_MIN_BLOCKS
#define CC1D_VEC_MIN_BLOCKS 1
#endif
constexpr int kVecV = CC1D_VEC_V;

// Linear single-token update with V contiguous channels per thread: x, bias,
// out are V-element runs, weights V*W, state V*(W-1) (state_len == W-1 and
// rows packed, so a thread's state is one contiguous run); every run moves
// as the widest aligned vectors that divide it.  All loads are independent
// (only the state row waits for the pool index).
// SCL: conv_state stored channel-last (unit channel stride): a thread's
// state is W-1 runs of V channels, one per position, ss_l apart.
// CIRC (channel-last only): circular buffer of any state_len S >= W-1; the
// window is the W-1 positions before cs = cache_seqlens[b] mod S and the new
// token is written at cs (one run instead of W-1).  cs is loaded alongside
// the pool index, so the state waits for one dependent round trip, as in the
// linear pooled case.
template <typename T, int W, bool SCL, bool CIRC = false>
__global__ void __launch_bounds__(128, CC1D_VEC_MIN_BLOCKS) update_vec_kernel(const UpdateArgs a) {
  static_assert(SCL || !CIRC, "circular mode is for channel-last states");
  griddep_wait();  // inputs and state may come from the previous kernel
  griddep_launch_dependents();
  constexpr int H = W - 1;
  constexpr int V = kVecV;
  constexpr int EX = vec_elems<T, V>();
  constexpr int EW = vec_elems<T, V * W>();
  constexpr int ES = vec_elems<T, V * H>();
  const i64 groups = a.D / V;
  const i64 b = blockIdx.y;  // grid (channel-group blocks, batch): no division
  const i64 g = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const i64 c0 = g * V;
  T* __restrict__ ob = static_cast<T*>(a.out) + b * a.os_b + c0;
  const int cs_raw = CIRC ? a.cache_seqlens[b] : 0;  // in flight with the pool index
  i64 row = b;
  if (a.idx != nullptr) {
    const int r = a.idx[b];
    if (r < 0 || r >= a.state_rows) {
      Pack<T, EX> z;
#pragma unroll
      for (int i = 0; i < EX; ++i) z.v[i] = Cvt<T>::to(0.f);
#pragma unroll
      for (int i = 0; i < V; i += EX) st_pack<T, EX>(ob + i, z);
      return;
    }
    row = r;
  }
  T* __restrict__ st = static_cast<T*>(a.state) + row * a.ss_b + (SCL ? c0 : c0 * a.S);
  T xv[V], bv[V], wv[V * W], sv[V * H];
  const T* __restrict__ xp = static_cast<const T*>(a.x) + b * a.xs_b + c0;
#pragma unroll
  for (int i = 0; i < V; i += EX) {
    const Pack<T, EX> px = ld_pack<T, EX>(xp + i);
#pragma unroll
    for (int e = 0; e < EX; ++e) xv[i + e] = px.v[e];
  }
  if (a.bias != nullptr) {
#pragma unroll
    for (int i = 0; i < V; i += EX) {
      const Pack<T, EX> pb = ld_pack<T, EX>(static_cast<const T*>(a.bias) + c0 + i);
#pragma unroll
      for (int e = 0; e < EX; ++e) bv[i + e] = pb.v[e];
    }
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) bv[i] = Cvt<T>::to(0.f);
  }
#pragma unroll
  for (int i = 0; i < V * W; i += EW) {
    const Pack<T, EW> pw = ld_pack<T, EW>(static_cast<const T*>(a.w) + c0 * W + i);
#pragma unroll
    for (int e = 0; e < EW; ++e) wv[i + e] = pw.v[e];
  }
  i64 cs = 0;  // circular write position
  if constexpr (SCL) {
    i64 ui = 0;  // circular: position of window slot j
    if constexpr (CIRC) {
      cs = (i64)cs_raw % a.S;
      if (cs < 0) cs += a.S;
      ui = cs - H;
      if (ui < 0) ui += a.S;
    }
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const T* sp = st + (CIRC ? ui : (i64)j) * a.ss_l;
#pragma unroll
      for (int i = 0; i < V; i += EX) {
        const Pack<T, EX> ps = ld_pack_rw<T, EX>(sp + i);
#pragma unroll
        for (int e = 0; e < EX; ++e) sv[(i + e) * H + j] = ps.v[e];
      }
      if constexpr (CIRC) ui = (ui + 1 == a.S) ? 0 : ui + 1;
    }
  } else {
#pragma unroll
    for (int i = 0; i < V * H; i += ES) {
      const Pack<T, ES> ps = ld_pack_rw<T, ES>(st + i);
#pragma unroll
      for (int e = 0; e < ES; ++e) sv[i + e] = ps.v[e];
    }
  }
  // Compute (same tap order and SiLU as every other kernel).
  Pack<T, EX> po[V / EX];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    float acc = Cvt<T>::f(bv[v]);
#pragma unroll
    for (int k = 0; k < H; ++k) acc = fmaf(Cvt<T>::f(wv[v * W + k]), Cvt<T>::f(sv[v * H + k]), acc);
    acc = fmaf(Cvt<T>::f(wv[v * W + H]), Cvt<T>::f(xv[v]), acc);
    if (a.silu) acc = silu_f(acc);
    po[v / EX].v[v % EX] = Cvt<T>::to(acc);
  }
#pragma unroll
  for (int i = 0; i < V; i += EX) st_pack<T, EX>(ob + i, po[i / EX]);
  if constexpr (CIRC) {
#pragma unroll
    for (int i = 0; i < V; i += EX) {
      Pack<T, EX> pn;
#pragma unroll
      for (int e = 0; e < EX; ++e) pn.v[e] = xv[i + e];
      st_pack<T, EX>(st + cs * a.ss_l + i, pn);
    }
  } else {
    // New rows [old[1..H-1], x] for the V channels, packed back to vectors.
    T nv[V * H];
#pragma unroll
    for (int v = 0; v < V; ++v) {
#pragma unroll
      for (int j = 0; j < H - 1; ++j) nv[v * H + j] = sv[v * H + j + 1];
      nv[v * H + H - 1] = xv[v];
    }
    if constexpr (SCL) {
#pragma unroll
      for (int j = 0; j < H; ++j) {
#pragma unroll
        for (int i = 0; i < V; i += EX) {
          Pack<T, EX> pn;
#pragma unroll
          for (int e = 0; e < EX; ++e) pn.v[e] = nv[(i + e) * H + j];
          st_pack<T, EX>(st + j * a.ss_l + i, pn);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < V * H; i += ES) {
        Pack<T, ES> pn;
#pragma unroll
        for (int e = 0; e < ES; ++e) pn.v[e] = nv[i + e];
        st_pack<T, ES>(st + i, pn);
      }
    }
  }
}

// Single-token circular-buffer decode (any strides, any state_len).  A warp
// owns 256 channels of one batch row, lane l the channels l + 32*v (v < 8), so
// every warp-wide access touches 32 consecutive channel rows.  All loads of a
// thread's 8 channels are issued before any store (no read-after-write
// ordering between channels); two dependent memory round trips per block.
template <typename T, int W>
__global__ void __launch_bounds__(128) update_circ_kernel(const UpdateArgs a) {
  constexpr int H = W - 1;
  constexpr int V = 8;
  constexpr int CHUNK = 128 * V;  // channels per block (4 warps x 256)
  const i64 chunks = ceil_div(a.D, (i64)CHUNK);
  const i64 b = blockIdx.x / chunks;
  const i64 cbase = (blockIdx.x - b * chunks) * CHUNK + (threadIdx.x >> 5) * 256 + (threadIdx.x & 31);
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ wt = static_cast<const T*>(a.w);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  T* __restrict__ out = static_cast<T*>(a.out);
  i64 row = b;
  if (a.idx != nullptr) {
    const int r = a.idx[b];
    if (r < 0 || r >= a.state_rows) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const i64 c = cbase + 32 * v;
        if (c < a.D) out[b * a.os_b + c * a.os_c] = Cvt<T>::to(0.f);
      }
      return;
    }
    row = r;
  }
  T* __restrict__ st = static_cast<T*>(a.state) + row * a.ss_b;
  i64 cs = (i64)a.cache_seqlens[b] % a.S;
  if (cs < 0) cs += a.S;
  i64 pos[H];
  {
    i64 ui = cs - H;
    if (ui < 0) ui += a.S;
#pragma unroll
    for (int j = 0; j < H; ++j) {
      pos[j] = ui * a.ss_l;
      ui = (ui + 1 == a.S) ? 0 : ui + 1;
    }
  }
  T xv[V];
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const i64 c = cbase + 32 * v;
    acc[v] = 0.f;
    xv[v] = Cvt<T>::to(0.f);
    if (c < a.D) {
      xv[v] = x[b * a.xs_b + c * a.xs_c];
      acc[v] = bias ? Cvt<T>::f(bias[c * a.bs]) : 0.f;
      const T* sc = st + c * a.ss_c;
#pragma unroll
      for (int k = 0; k < H; ++k) acc[v] = fmaf(Cvt<T>::f(wt[c * a.ws_c + k * a.ws_k]), Cvt<T>::f(sc[pos[k]]), acc[v]);
      acc[v] = fmaf(Cvt<T>::f(wt[c * a.ws_c + H * a.ws_k]), Cvt<T>::f(xv[v]), acc[v]);
    }
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const i64 c = cbase + 32 * v;
    if (c < a.D) {
      float o = acc[v];
      if (a.silu) o = silu_f(o);
      out[b * a.os_b + c * a.os_c] = Cvt<T>::to(o);
      st[c * a.ss_c + cs * a.ss_l] = xv[v];
    }
  }
}

// Element `i` of a state row held in NW 32-bit words (selects, no local
// memory; the word predicates depend only on i, so they are shared by all
// channels of a thread).
template <typename T, int NW>
__device__ __forceinline__ float row_elem(const uint32_t (&w)[NW], int i) {
  const int wi = (i * (int)sizeof(T)) >> 2;
  uint32_t word = w[0];
#pragma unroll
  for (int k = 1; k < NW; ++k) word = wi == k ? w[k] : word;
  if (sizeof(T) == 4) return bits_to_float<T>(word);
  return bits_to_float<T>((i & 1) ? (word >> 16) : (word & 0xffffu));
}

// W weights of one channel as floats: one vector load when they are
// contiguous and the vector is 4, 8 or 16 bytes, else W scalar loads.
template <typename T, int W>
__device__ __forceinline__ void load_taps(const T* __restrict__ p, i64 ws_k, bool vec, float (&w)[W]) {
  constexpr int BYTES = W * (int)sizeof(T);
  if constexpr (BYTES == 4 || BYTES == 8 || BYTES == 16) {
    if (vec) {
      const Pack<T, W> pk = ld_pack<T, W>(p);
#pragma unroll
      for (int k = 0; k < W; ++k) w[k] = Cvt<T>::f(pk.v[k]);
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < W; ++k) w[k] = Cvt<T>::f(p[k * ws_k]);
}

// Circular-buffer decode step (seqlen 1, cache_seqlens given) for state rows
// of 16 or 32 bytes with unit element stride.  Each channel's whole row is
// fetched with one or two 16-byte loads that do not wait for the buffer
// position (nor for anything but the pool index), so the position load, the
// rows, x, weight and bias are all in flight together -- one memory round
// trip instead of two.  The W-1 window is then picked from registers.
// Warps are mapped flat onto (batch row, range of 32*V channels), lane l
// taking channels l, l+32, ..., so a warp's row load covers 32 consecutive
// channel rows (512 or 1024 contiguous bytes) and no warp straddles two
// batch rows.  Addresses advance by precomputed pointer steps.  Same
// arithmetic order as update_circ_kernel.
// Few channels per lane and a full SM of warps beat deep per-thread batches
// here (B200, C3b shape: 2 / 16 -> 12.5 us; 8 / none -> 22.7 us): the
// kernel is bound by memory latency, not by instruction count.
#ifndef CC1D_CIRC_V16
#define CC1D_CIRC_V16 2  // channels per lane for 16-byte rows (half that for 32-byte rows)
#endif
#ifndef CC1D_CIRC_MIN_BLOCKS
#define CC1D_CIRC_MIN_BLOCKS 16
#endif
template <int NW>
constexpr int circ_lane_channels() {
  return NW == 4 ? CC1D_CIRC_V16 : (CC1D_CIRC_V16 / 2 > 0 ? CC1D_CIRC_V16 / 2 : 1);
}

template <typename T, int W, int NW>
__global__ void __launch_bounds__(128, CC1D_CIRC_MIN_BLOCKS) update_circ_row_kernel(const UpdateArgs a,
                                                                                   const int warps_per_row,
                                                                                   const bool taps_vec) {
  griddep_wait();  // inputs and state may come from the previous kernel
  griddep_launch_dependents();
  constexpr int H = W - 1;
  constexpr int V = circ_lane_channels<NW>();  // channels per lane
  // Grid (warp groups of a batch row, batch): no division.
  const int wr = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5));
  if (wr >= warps_per_row) return;
  const i64 b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const i64 c0 = (i64)wr * (32 * V) + lane;
  const int nv = c0 >= a.D ? 0 : (int)min((i64)V, (a.D - c0 + 31) >> 5);  // channels of this lane in range
  T* __restrict__ out = static_cast<T*>(a.out) + b * a.os_b + c0 * a.os_c;
  const i64 out_step = 32 * a.os_c;
  i64 row = b;
  if (a.idx != nullptr) {
    const int r = a.idx[b];
    if (r < 0 || r >= a.state_rows) {
#pragma unroll
      for (int v = 0; v < V; ++v)
        if (v < nv) out[v * out_step] = Cvt<T>::to(0.f);
      return;
    }
    row = r;
  }
  T* __restrict__ st = static_cast<T*>(a.state) + row * a.ss_b + c0 * a.ss_c;
  const i64 st_step = 32 * a.ss_c;
  const T* __restrict__ xp = static_cast<const T*>(a.x) + b * a.xs_b + c0 * a.xs_c;
  const i64 x_step = 32 * a.xs_c;
  const T* __restrict__ wp = static_cast<const T*>(a.w) + c0 * a.ws_c;
  const i64 w_step = 32 * a.ws_c;
  const T* __restrict__ bp = a.bias ? static_cast<const T*>(a.bias) + c0 * a.bs : nullptr;
  const i64 b_step = 32 * a.bs;
  const int cs_raw = a.cache_seqlens[b];
  uint32_t rw[V][NW];
  T xv[V];
  float wv[V][W];
  float acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    if (v < nv) {
      const uint4* src = reinterpret_cast<const uint4*>(st + v * st_step);
#pragma unroll
      for (int q = 0; q < NW / 4; ++q) {
        const uint4 u = src[q];
        rw[v][4 * q + 0] = u.x;
        rw[v][4 * q + 1] = u.y;
        rw[v][4 * q + 2] = u.z;
        rw[v][4 * q + 3] = u.w;
      }
      xv[v] = xp[v * x_step];
      load_taps<T, W>(wp + v * w_step, a.ws_k, taps_vec, wv[v]);
      acc[v] = bp ? Cvt<T>::f(bp[v * b_step]) : 0.f;
    }
  }
  int cs = cs_raw % (int)a.S;  // state_len is a few elements: 32-bit arithmetic
  if (cs < 0) cs += (int)a.S;
  int pos[H];
  {
    int ui = cs - H;
    if (ui < 0) ui += (int)a.S;
#pragma unroll
    for (int j = 0; j < H; ++j) {
      pos[j] = ui;
      ui = (ui + 1 == (int)a.S) ? 0 : ui + 1;
    }
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    if (v < nv) {
#pragma unroll
      for (int k = 0; k < H; ++k) acc[v] = fmaf(wv[v][k], row_elem<T, NW>(rw[v], pos[k]), acc[v]);
      acc[v] = fmaf(wv[v][H], Cvt<T>::f(xv[v]), acc[v]);
      float o = acc[v];
      if (a.silu) o = silu_f(o);
      out[v * out_step] = Cvt<T>::to(o);
      st[v * st_step + cs] = xv[v];
    }
  }
}

// One state slot of one sequence: states[i, c, j] for the channels of this
// block.  Grid (channel blocks, slot j, sequence i): no index division.
template <typename T>
__device__ __forceinline__ void varlen_slot(const VarlenArgs& a, i64 i, i64 j, i64 c) {
  const i64 beg = a.cu[i];
  const i64 end = a.cu[i + 1];
  const i64 start = max(beg, end - a.S);
  const i64 cnt = end - start;
  T v = Cvt<T>::to(0.f);
  const i64 tok = end - a.S + j;
  if (cnt > 0 && j >= a.S - cnt && tok >= 0 && tok < a.total_tokens)
    v = static_cast<const T*>(a.x)[tok * a.xs_t + c * a.xs_c];
  static_cast<T*>(a.st)[i * a.ss_b + c * a.ss_c + j * a.ss_l] = v;
}

template <typename T>
__global__ void __launch_bounds__(256) varlen_states_kernel(const VarlenArgs a) {
  griddep_wait();  // x and cu_seqlens may come from the previous kernel
  griddep_launch_dependents();
  const i64 c = (i64)blockIdx.x * blockDim.x + threadIdx.x;
  if (c < a.D) varlen_slot<T>(a, blockIdx.z, blockIdx.y, c);
}

// More sequences or slots than a grid's y/z extent: flat index (divisions).
template <typename T>
__global__ void varlen_states_flat_kernel(const VarlenArgs a) {
  const i64 n = a.B * a.S * a.D;
  for (i64 e = (i64)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (i64)gridDim.x * blockDim.x) {
    const i64 bj = e / a.D;
    varlen_slot<T>(a, bj / a.S, bj % a.S, e - bj * a.D);
  }
}

// Update supports widths 2..9 for every dtype (no lane-vector halo).
template <typename T, typename F>
cudaError_t dispatch_update_width(int width, F&& f) {
  switch (width) {
    case 2: return f.template operator()<T, 2>();
    case 3: return f.template operator()<T, 3>();
    case 4: return f.template operator()<T, 4>();
    case 5: return f.template operator()<T, 5>();
    case 6: return f.template operator()<T, 6>();
    case 7: return f.template operator()<T, 7>();
    case 8: return f.template operator()<T, 8>();
    case 9: return f.template operator()<T, 9>();
    default: return cudaErrorInvalidValue;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool aligned_bytes(const void* p, i64 bytes) { return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)bytes) == 0; }

// Conditions of update_vec_kernel: one new token, (D, W) contiguous
// weights, unit channel stride for x / out / bias, D a multiple of the
// channels per thread, and every run aligned to the vector that moves it.
// Returns 1 for linear mode with packed state rows (state_len == W-1, stride
// 1 over state_len, rows back to back), 2 for linear mode with a channel-last
// state (state_len == W-1, unit channel stride), 3 for circular mode with a
// channel-last state (any state_len), 0 when the kernel does not apply
// (circular packed rows go to update_circ_row_kernel).
template <typename T, int W>
int vec_path(const UpdateArgs& a) {
  constexpr int V = kVecV;
  constexpr i64 esz = (i64)sizeof(T);
  constexpr i64 EX = vec_elems<T, V>(), EW = vec_elems<T, V * W>(), ES = vec_elems<T, V * (W - 1)>();
  const bool common = a.L == 1 && a.D % V == 0 && a.ws_k == 1 && a.ws_c == W && aligned_bytes(a.w, EW * esz) &&
                      a.xs_c == 1 && aligned_bytes(a.x, EX * esz) && (a.B == 1 || a.xs_b % EX == 0) &&
                      a.os_c == 1 && aligned_bytes(a.out, EX * esz) && (a.B == 1 || a.os_b % EX == 0) &&
                      (a.bias == nullptr || (a.bs == 1 && aligned_bytes(a.bias, EX * esz)));
  if (!common) return 0;
  const bool chanlast = a.ss_c == 1 && aligned_bytes(a.state, EX * esz) && a.ss_l % EX == 0 && a.ss_b % EX == 0;
  if (a.cache_seqlens != nullptr) return chanlast ? 3 : 0;
  if (a.S != W - 1) return 0;
  if (a.ss_l == 1 && a.ss_c == a.S && aligned_bytes(a.state, ES * esz) && a.ss_b % ES == 0) return 1;
  return chanlast ? 2 : 0;
}

// Circular rows of 16 or 32 bytes, unit element stride, 16-byte aligned:
// returns the row size in 32-bit words (4 or 8), else 0.
template <typename T>
int circ_row_words(const UpdateArgs& a) {
  if (a.cache_seqlens == nullptr || a.L != 1 || a.ss_l != 1 || !aligned16(a.state)) return 0;
  const i64 esz = (i64)sizeof(T);
  const i64 row_bytes = a.S * esz;
  if (row_bytes != 16 && row_bytes != 32) return 0;
  if ((a.ss_c * esz) % 16 != 0 || (a.ss_b * esz) % 16 != 0) return 0;
  return (int)(row_bytes / 4);
}

struct LaunchUpdate {
  const UpdateArgs& a;
  cudaStream_t stream;
  template <typename T, int W>
  cudaError_t operator()() {
    const int threads = 128;
    const int vp = a.B <= 65535 ? vec_path<T, W>(a) : 0;
    if (vp != 0) {
      const dim3 grid((unsigned)ceil_div(a.D / kVecV, (i64)threads), (unsigned)a.B);
      if (vp == 3) return launch_pdl(update_vec_kernel<T, W, true, true>, grid, dim3(threads), 0, stream, a);
      if (vp == 2) return launch_pdl(update_vec_kernel<T, W, true>, grid, dim3(threads), 0, stream, a);
      return launch_pdl(update_vec_kernel<T, W, false>, grid, dim3(threads), 0, stream, a);
    }
    const int nw = a.B <= 65535 ? circ_row_words<T>(a) : 0;
    if (nw == 4 || nw == 8) {
      const int V = nw == 4 ? circ_lane_channels<4>() : circ_lane_channels<8>();
      const i64 warps_per_row = ceil_div(a.D, (i64)32 * V);
      if (warps_per_row > 0x7fffffffLL || a.B > 65535) return cudaErrorInvalidConfiguration;
      const dim3 blocks((unsigned)ceil_div(warps_per_row, (i64)threads / 32), (unsigned)a.B);
      const i64 tb = W * (i64)sizeof(T);
      const bool taps_vec = a.ws_k == 1 && (tb == 4 || tb == 8 || tb == 16) && (a.ws_c * (i64)sizeof(T)) % tb == 0 &&
                            (reinterpret_cast<uintptr_t>(a.w) % (uintptr_t)tb) == 0;
      if (nw == 4)
        return launch_pdl(update_circ_row_kernel<T, W, 4>, blocks, dim3(threads), 0, stream, a, (int)warps_per_row,
                          taps_vec);
      return launch_pdl(update_circ_row_kernel<T, W, 8>, blocks, dim3(threads), 0, stream, a, (int)warps_per_row,
                        taps_vec);
    }
    if (a.cache_seqlens != nullptr && a.L == 1) {
      const i64 blocks = ceil_div(a.D, (i64)threads * 8) * a.B;
      if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
      update_circ_kernel<T, W><<<(unsigned)blocks, threads, 0, stream>>>(a);
      return cudaGetLastError();
    }
    if (a.cache_seqlens == nullptr && a.L >= 1 && a.L <= kLinLMax && a.S <= kLinSMax && a.B <= 65535) {
      const dim3 grid((unsigned)ceil_div(a.D, (i64)threads), (unsigned)a.B);
      if (a.S == W - 1) {
        switch (a.L) {
          case 1: return launch_pdl(update_lin_kernel<T, W, W - 1, 1>, grid, dim3(threads), 0, stream, a);
          case 2: return launch_pdl(update_lin_kernel<T, W, W - 1, 2>, grid, dim3(threads), 0, stream, a);
          case 3: return launch_pdl(update_lin_kernel<T, W, W - 1, 3>, grid, dim3(threads), 0, stream, a);
          case 4: return launch_pdl(update_lin_kernel<T, W, W - 1, 4>, grid, dim3(threads), 0, stream, a);
          default: break;
        }
      }
      return launch_pdl(update_lin_kernel<T, W, 0, 0>, grid, dim3(threads), 0, stream, a);
    }
    const i64 blocks = ceil_div(a.D, (i64)threads) * a.B;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    update_kernel<T, W><<<(unsigned)blocks, threads, 0, stream>>>(a);
    return cudaGetLastError();
  }
};

}  // namespace

cudaError_t launch_update(int dtype, int width, const UpdateArgs& a, cudaStream_t stream) {
  if (a.B == 0 || a.D == 0) return cudaSuccess;
  LaunchUpdate f{a, stream};
  switch (dtype) {
    case 0: return dispatch_update_width<__half>(width, f);
    case 1: return dispatch_update_width<__nv_bfloat16>(width, f);
    case 2: return dispatch_update_width<float>(width, f);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_varlen_states(int dtype, const VarlenArgs& a, cudaStream_t stream) {
  const i64 n = a.B * a.S * a.D;
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  if (a.B <= 65535 && a.S <= 65535 && ceil_div(a.D, (i64)threads) <= 0x7fffffffLL) {
    const dim3 grid((unsigned)ceil_div(a.D, (i64)threads), (unsigned)a.S, (unsigned)a.B);
    switch (dtype) {
      case 0: return launch_pdl(varlen_states_kernel<__half>, grid, dim3(threads), 0, stream, a);
      case 1: return launch_pdl(varlen_states_kernel<__nv_bfloat16>, grid, dim3(threads), 0, stream, a);
      case 2: return launch_pdl(varlen_states_kernel<float>, grid, dim3(threads), 0, stream, a);
      default: return cudaErrorInvalidValue;
    }
  }
  const unsigned blocks = (unsigned)std::min<i64>(ceil_div(n, threads), 1 << 20);
  switch (dtype) {
    case 0: varlen_states_flat_kernel<__half><<<blocks, threads, 0, stream>>>(a); break;
    case 1: varlen_states_flat_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(a); break;
    case 2: varlen_states_flat_kernel<float><<<blocks, threads, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace cc1d
