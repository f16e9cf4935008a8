// Device-side helpers shared by the kernels: scalar conversions, 16-byte
// vector I/O, warp/block reductions and activation functions.  Depends only
// on the CUDA headers (no PyTorch), so allocation-free entry points can use it.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tb {

// ---- scalar conversions ----------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// ---- 16-byte vectors ---------------------------------------------------------
// VecT<T>::N elements of T packed in one 16-byte word.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T v[N];
  };
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&out)[16 / sizeof(T)]) {
  Vec16<T> t;
  t.raw = *reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) out[i] = to_f<T>(t.v[i]);
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float (&in)[16 / sizeof(T)]) {
  Vec16<T> t;
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) t.v[i] = from_f<T>(in[i]);
  *reinterpret_cast<uint4*>(p) = t.raw;
}

// ---- reductions --------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}

// ---- activations (math written from the definitions) -------------------------
// fast-division sigmoid: __fdividef returns 0 once the denominator overflows,
// which is the correct limit for large negative x
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float silu_(float x) { return x * sigmoidf_(x); }
__device__ __forceinline__ float silu_grad_(float x) {
  float s = sigmoidf_(x);
  return s * (1.f + x * (1.f - s));
}
// exact GELU (erf form) and its derivative
__device__ __forceinline__ float gelu_(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float gelu_grad_(float x) {
  return 0.5f * (1.f + erff(x * 0.70710678118654752f)) + x * 0.39894228040143268f * __expf(-0.5f * x * x);
}

enum Act : int { ACT_SILU = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_NONE = 3 };

__device__ __forceinline__ float act_f(int a, float x) {
  switch (a) {
    case ACT_SILU: return silu_(x);
    case ACT_GELU: return gelu_(x);
    case ACT_RELU: return fmaxf(x, 0.f);
    default: return x;
  }
}
__device__ __forceinline__ float act_grad_f(int a, float x) {
  switch (a) {
    case ACT_SILU: return silu_grad_(x);
    case ACT_GELU: return gelu_grad_(x);
    case ACT_RELU: return x > 0.f ? 1.f : 0.f;
    default: return 1.f;
  }
}

}  // namespace tb
