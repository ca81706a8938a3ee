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

// SiLU(v) = v * sigmoid(v), evaluated with the fast exp and divide
// intrinsics (the op is SFU-bound otherwise).
__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// d SiLU / dv = s * (1 + v * (1 - s)) with s = sigmoid(v).
__device__ __forceinline__ float silu_grad_f(float v) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-v));
  return s * (1.0f + v * (1.0f - s));
}

__host__ __device__ __forceinline__ i64 ceil_div(i64 a, i64 b) { return (a + b - 1) / b; }

}  // namespace cc1d
