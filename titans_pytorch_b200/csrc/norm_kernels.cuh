// RMSNorm backward kernels, shared by the PyTorch-facing entry point
// (norm.cu) and the allocation-free C entry point (noalloc.cu).
//
// rms_bwd_kernel: one warp per row; lane owns CH 16-byte chunks; writes dx and
// (when dw_part is non-null) one row of per-block column partial sums of
// dy * xhat into dw_part[blockIdx.x * D .. + D) -- every column of that row is
// written, so the partial buffer needs no clearing.  colsum_kernel then sums
// the G partial rows in a fixed order (deterministic).
#pragma once

#include "device_common.cuh"

namespace tb {

template <typename T, int CH>
__global__ void __launch_bounds__(256) rms_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                      const T* __restrict__ w, const float* __restrict__ rstd,
                                                      T* __restrict__ dx, float* __restrict__ dw_part,
                                                      int64_t rows, int D, const T* __restrict__ dadd = nullptr) {
  constexpr int V = Vec16<T>::N;
  extern __shared__ float smem[];  // [nwarps][D]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t warp0 = (int64_t)blockIdx.x * nw + wid;
  const int64_t nwarps = (int64_t)gridDim.x * nw;
  float acc[CH][V];
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int i = 0; i < V; ++i) acc[c][i] = 0.f;

  for (int64_t r = warp0; r < rows; r += nwarps) {
    const T* dyr = dy + r * D;
    const T* xr = x + r * D;
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        float a[V], b[V], ww[V];
        load16<T>(dyr + col, a);
        load16<T>(xr + col, b);
        load16<T>(w + col, ww);
#pragma unroll
        for (int i = 0; i < V; ++i) dot += a[i] * ww[i] * b[i];
      }
    }
    dot = warp_sum(dot) * rs * rs / (float)D;
    T* dxr = dx + r * D;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        float a[V], b[V], ww[V], o[V];
        load16<T>(dyr + col, a);
        load16<T>(xr + col, b);
        load16<T>(w + col, ww);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          o[i] = rs * (a[i] * ww[i] - b[i] * dot);
          acc[c][i] += a[i] * b[i] * rs;
        }
        if (dadd != nullptr) {  // gradient arriving at the normalised input directly (fused residual add)
          float e[V];
          load16<T>(dadd + r * D + col, e);
#pragma unroll
          for (int i = 0; i < V; ++i) o[i] += e[i];
        }
        store16<T>(dxr + col, o);
      }
    }
  }
  if (dw_part == nullptr) return;
  // reduce the per-warp column partials through shared memory
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * V;
    if (col < D)
#pragma unroll
      for (int i = 0; i < V; ++i) smem[wid * D + col + i] = acc[c][i];
  }
  __syncthreads();
  for (int col = threadIdx.x; col < D; col += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < nw; ++k) s += smem[k * D + col];
    dw_part[(int64_t)blockIdx.x * D + col] = s;
  }
}

// Column sums of a [G, D] fp32 partial buffer (fixed order).
static __global__ void colsum_kernel(const float* __restrict__ part, float* __restrict__ out, int G, int D) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= D) return;
  float s = 0.f;
  for (int g = 0; g < G; ++g) s += part[(int64_t)g * D + col];
  out[col] = s;
}

// The same column sums with more parallelism: block = 32 columns x 16 row
// groups; each thread sums every 16th partial row of its column, then the 16
// group sums are added in a fixed order (deterministic).
static __global__ void colsum_par_kernel(const float* __restrict__ part, float* __restrict__ out, int G, int D) {
  __shared__ float red[16][33];
  const int col = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (col < D)
    for (int g = threadIdx.y; g < G; g += 16) s += part[(int64_t)g * D + col];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && col < D) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += red[k][threadIdx.x];
    out[col] = t;
  }
}

}  // namespace tb
