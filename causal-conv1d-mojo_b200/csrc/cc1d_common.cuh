// Shared device helpers for the sm_100a causal depthwise conv1d kernels.
//
// Every kernel reads its input dtype (fp16 / bf16 / fp32), accumulates in
// fp32 and rounds once on store.  The conv tap order (bias first, then taps
// k = 0..W-1 through fmaf) is the same in the forward, backward-recompute
// and decode-update kernels, so a decode loop reproduces a full forward
// bit-for-bit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cc1d {

typedef int64_t i64;

constexpr unsigned kFull = 0xffffffffu;
// Sequence id used for positions outside [0, L); never equal to a real id
// of a position whose value matters (values there are zero).
constexpr int kNoSeq = (int)0x80000000;

// Programmatic dependent launch (kernels started with launch_pdl): wait
// until the previous kernel in the stream has completed and its memory is
// visible (a no-op for a normal launch); and let the next kernel be
// scheduled once every block of this one has signalled or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename T>
struct Cvt;
template <>
struct Cvt<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float to(float v) { return v; }
};
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 to(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half to(float v) { return __float2half_rn(v); }
};

// N consecutive elements moved as one aligned vector access of
// N*sizeof(T) bytes (2, 4, 8 or 16).
template <int BYTES>
struct RawT;
template <>
struct RawT<16> { typedef uint4 type; };
template <>
struct RawT<8> { typedef uint2 type; };
template <>
struct RawT<4> { typedef unsigned int type; };
template <>
struct RawT<2> { typedef unsigned short type; };

template <typename T, int N>
struct Pack {
  typedef typename RawT<N * sizeof(T)>::type Raw;
  union {
    Raw raw;
    T v[N];
  };
};

template <typename T, int N>
__device__ __forceinline__ Pack<T, N> ld_pack(const T* __restrict__ p) {
  Pack<T, N> pk;
  pk.raw = __ldg(reinterpret_cast<const typename Pack<T, N>::Raw*>(p));
  return pk;
}

template <typename T, int N>
__device__ __forceinline__ void st_pack(T* __restrict__ p, const Pack<T, N>& pk) {
  *reinterpret_cast<typename Pack<T, N>::Raw*>(p) = pk.raw;
}

// Load N elements p[i*stride] for i < n (the rest read as 0).  VEC means
// stride 1 and p aligned to N*sizeof(T): one vector load when all N are valid.
template <typename T, int N, bool VEC>
__device__ __forceinline__ void load_strided(const T* __restrict__ p, i64 stride, int n, float (&out)[N]) {
  if (VEC && n == N) {
    const Pack<T, N> pk = ld_pack<T, N>(p);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = Cvt<T>::f(pk.v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = (i < n) ? Cvt<T>::f(p[VEC ? (i64)i : (i64)i * stride]) : 0.f;
  }
}

template <typename T, int N, bool VEC>
__device__ __forceinline__ void store_strided(T* __restrict__ p, i64 stride, int n, const float (&v)[N]) {
  if (VEC && n == N) {
    Pack<T, N> pk;
#pragma unroll
    for (int i = 0; i < N; ++i) pk.v[i] = Cvt<T>::to(v[i]);
    st_pack<T, N>(p, pk);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < n) p[VEC ? (i64)i : (i64)i * stride] = Cvt<T>::to(v[i]);
  }
}

// SiLU(v) = v * sigmoid(v), sigmoid(v) = 1 / (1 + exp(-v)) with
// exp(-v) = 2^(-v * log2(e)), each step one hardware instruction: the
// approximate base-2 exponential (ex2.approx, rel. error ~2^-22) and the
// approximate reciprocal (rcp.approx, ~1 ulp).  At v << 0, 2^(...) = inf and
// the reciprocal is 0, so SiLU -> -0 and SiLU' -> 0.  Every kernel (scalar or
// packed) evaluates exactly this sequence, so the forward, the decode update
// and the backward recomputation agree bit for bit.
constexpr float kNegLog2e = -1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

__device__ __forceinline__ float sigmoid_f(float v) { return rcp_approx(1.0f + ex2_approx(v * kNegLog2e)); }
__device__ __forceinline__ float silu_f(float v) { return v * sigmoid_f(v); }

// d SiLU / dv = s * (1 + v * (1 - s)) with s = sigmoid(v).
__device__ __forceinline__ float silu_grad_f(float v) {
  const float s = sigmoid_f(v);
  return s * fmaf(v, fmaf(s, -1.0f, 1.0f), 1.0f);
}

// ---- two adjacent channels per thread, packed fp32 math (sm_100 FFMA2) ----

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

__device__ __forceinline__ float2 sigmoid2(float2 v) {
  const float2 t = mul2(v, f2(kNegLog2e, kNegLog2e));
  const float2 d = add2(f2(1.0f, 1.0f), f2(ex2_approx(t.x), ex2_approx(t.y)));
  return f2(rcp_approx(d.x), rcp_approx(d.y));
}
__device__ __forceinline__ float2 silu2(float2 v) { return mul2(v, sigmoid2(v)); }
__device__ __forceinline__ float2 silu_grad2(float2 v) {
  const float2 s = sigmoid2(v);
  const float2 one = f2(1.0f, 1.0f);
  return mul2(s, fma2(v, fma2(s, f2(-1.0f, -1.0f), one), one));
}

// Storage word of two adjacent elements and its conversion to/from float2.
template <typename T>
struct Pair;
template <>
struct Pair<__nv_bfloat16> {
  typedef uint32_t W;
  static __device__ __forceinline__ float2 unpack(W w) {
    return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  static __device__ __forceinline__ W pack(float2 v) {
    __nv_bfloat162 h = __float22bfloat162_rn(v);
    return *reinterpret_cast<W*>(&h);
  }
};
template <>
struct Pair<__half> {
  typedef uint32_t W;
  static __device__ __forceinline__ float2 unpack(W w) { return __half22float2(*reinterpret_cast<__half2*>(&w)); }
  static __device__ __forceinline__ W pack(float2 v) {
    __half2 h = __float22half2_rn(v);
    return *reinterpret_cast<W*>(&h);
  }
};
template <>
struct Pair<float> {
  typedef float2 W;
  static __device__ __forceinline__ float2 unpack(W w) { return w; }
  static __device__ __forceinline__ W pack(float2 v) { return v; }
};

__host__ __device__ __forceinline__ i64 ceil_div(i64 a, i64 b) { return (a + b - 1) / b; }

}  // namespace cc1d
