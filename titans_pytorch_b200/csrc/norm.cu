// RMSNorm forward/backward.  One warp owns one row; each lane holds CH
// 16-byte chunks of the row, so x is read from HBM once in the forward.
// The backward writes per-block partial column sums of dy*xhat (the weight
// gradient), reduced by a second small kernel in a fixed order
// (deterministic, no atomics).
#include "common.cuh"
#include "norm_kernels.cuh"

namespace tb {

template <typename T, int CH>
__global__ void __launch_bounds__(256) rms_fwd_kernel(const T* __restrict__ x, int64_t xs,
                                                      const T* __restrict__ w, T* __restrict__ y,
                                                      float* __restrict__ rstd, int64_t rows, int D,
                                                      float eps) {
  constexpr int V = Vec16<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const T* xr = x + r * xs;
    float v[CH][V];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        load16<T>(xr + col, v[c]);
#pragma unroll
        for (int i = 0; i < V; ++i) ss += v[c][i] * v[c][i];
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
    T* yr = y + r * (int64_t)D;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        float wv[V];
        load16<T>(w + col, wv);
#pragma unroll
        for (int i = 0; i < V; ++i) v[c][i] = v[c][i] * rs * wv[i];
        store16<T>(yr + col, v[c]);
      }
    }
    if (lane == 0) rstd[r] = rs;
  }
}

// h = x + r (rounded to T, as the unfused add is) and y = rmsnorm(h) * w in
// one pass: residual add fused into the normalisation
template <typename T, int CH>
__global__ void __launch_bounds__(256) rms_add_fwd_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                          T* __restrict__ h, const T* __restrict__ w,
                                                          T* __restrict__ y, float* __restrict__ rstd, int64_t rows,
                                                          int D, float eps) {
  constexpr int V = Vec16<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = warp0; r < rows; r += nwarps) {
    float v[CH][V];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        float a[V];
        load16<T>(x + r * D + col, v[c]);
        load16<T>(res + r * D + col, a);
#pragma unroll
        for (int i = 0; i < V; ++i) v[c][i] = to_f<T>(from_f<T>(v[c][i] + a[i]));
        store16<T>(h + r * D + col, v[c]);
#pragma unroll
        for (int i = 0; i < V; ++i) ss += v[c][i] * v[c][i];
      }
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * V;
      if (col < D) {
        float wv[V];
        load16<T>(w + col, wv);
#pragma unroll
        for (int i = 0; i < V; ++i) v[c][i] = v[c][i] * rs * wv[i];
        store16<T>(y + r * D + col, v[c]);
      }
    }
    if (lane == 0) rstd[r] = rs;
  }
}

template <typename T, int CH>
static void launch_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, float eps) {
  const int64_t rows = x.size(0);
  const int D = x.size(1);
  const int threads = 256;
  int64_t blocks = std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 8);
  blocks = std::max<int64_t>(blocks, 1);
  rms_fwd_kernel<T, CH><<<blocks, threads, 0, stream()>>>(
      (const T*)x.data_ptr(), x.stride(0), (const T*)w.data_ptr(), (T*)y.data_ptr(),
      rstd.data_ptr<float>(), rows, D, eps);
}

template <typename T, int CH>
static void launch_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                       at::Tensor& dx, float* dw_part, int blocks, const T* dadd = nullptr) {
  const int64_t rows = x.size(0);
  const int D = x.size(1);
  const int threads = 256;
  size_t smem = dw_part ? (size_t)(threads / 32) * D * sizeof(float) : 0;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(rms_bwd_kernel<T, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rms_bwd_kernel<T, CH><<<blocks, threads, smem, stream()>>>(
      (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)w.data_ptr(), rstd.data_ptr<float>(),
      (T*)dx.data_ptr(), dw_part, rows, D, dadd);
}

#define TB_CH_SWITCH(CHN, ...)                          \
  switch (CHN) {                                        \
    case 1: { constexpr int CH = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int CH = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int CH = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int CH = 4; __VA_ARGS__; break; } \
    case 5: case 6: { constexpr int CH = 6; __VA_ARGS__; break; } \
    case 7: case 8: { constexpr int CH = 8; __VA_ARGS__; break; } \
    default: { constexpr int CH = 16; __VA_ARGS__; break; } \
  }

std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, double eps) {
  TB_CHECK_CUDA(x);
  TB_CHECK_LASTDIM(x);
  TORCH_CHECK(x.dim() == 2, "rms_norm_fwd: x must be 2-D");
  const at::cuda::CUDAGuard g(x.device());
  const int D = x.size(1);
  at::Tensor wc = contig16(w.to(x.scalar_type()));
  at::Tensor y = at::empty({x.size(0), D}, x.options());
  at::Tensor rstd = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  if (x.size(0) == 0) return {y, rstd};
  TB_DISPATCH_FLOAT(x.scalar_type(), "rms_norm_fwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(D % V == 0 && (x.stride(0) % V) == 0 && ((uintptr_t)x.data_ptr() % 16) == 0,
                "rms_norm_fwd: D and row stride must be multiples of ", V);
    const int chn = (D + 32 * V - 1) / (32 * V);
    TORCH_CHECK(chn <= 16, "rms_norm_fwd: D too large");
    TB_CH_SWITCH(chn, launch_fwd<scalar_t, CH>(x, wc, y, rstd, (float)eps));
  });
  check_launch("rms_norm_fwd");
  return {y, rstd};
}

std::vector<at::Tensor> rms_norm_add_fwd(const at::Tensor& x, const at::Tensor& res, const at::Tensor& w,
                                         double eps) {
  TB_CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.sizes() == res.sizes() && x.is_contiguous() && res.is_contiguous() &&
                  x.scalar_type() == res.scalar_type() && aligned16(x) && aligned16(res),
              "rms_norm_add_fwd: x and residual must be contiguous [rows, D] of one dtype");
  const at::cuda::CUDAGuard g(x.device());
  const int D = x.size(1);
  const int64_t rows = x.size(0);
  at::Tensor wc = contig16(w.to(x.scalar_type()));
  at::Tensor h = at::empty_like(x), y = at::empty_like(x);
  at::Tensor rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {h, y, rstd};
  TB_DISPATCH_FLOAT(x.scalar_type(), "rms_norm_add_fwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(D % V == 0, "rms_norm_add_fwd: D must be a multiple of ", V);
    const int chn = (D + 32 * V - 1) / (32 * V);
    TORCH_CHECK(chn <= 16, "rms_norm_add_fwd: D too large");
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 8));
    TB_CH_SWITCH(chn, rms_add_fwd_kernel<scalar_t, CH><<<blocks, 256, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (const scalar_t*)res.data_ptr(), (scalar_t*)h.data_ptr(),
        (const scalar_t*)wc.data_ptr(), (scalar_t*)y.data_ptr(), rstd.data_ptr<float>(), rows, D, (float)eps));
  });
  check_launch("rms_norm_add_fwd");
  return {h, y, rstd};
}

std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                     const at::Tensor& rstd, bool need_dw, const c10::optional<at::Tensor>& dadd) {
  TB_CHECK_CUDA(x);
  const at::cuda::CUDAGuard g(x.device());
  at::Tensor xc = contig16(x), dyc = contig16(dy);
  const int D = x.size(1);
  const int64_t rows = x.size(0);
  at::Tensor wc = contig16(w.to(x.scalar_type()));
  at::Tensor dx = at::empty_like(xc);
  at::Tensor dw = need_dw ? at::empty({D}, x.options().dtype(at::kFloat)) : at::empty({0}, x.options());
  if (rows == 0) {
    if (need_dw) dw.zero_();
    return {dx, dw};
  }
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 3));
  at::Tensor part = need_dw ? at::empty({blocks, D}, x.options().dtype(at::kFloat)) : at::Tensor();
  TB_DISPATCH_FLOAT(x.scalar_type(), "rms_norm_bwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(D % V == 0, "rms_norm_bwd: D must be a multiple of ", V);
    const int chn = (D + 32 * V - 1) / (32 * V);
    const scalar_t* da = nullptr;
    if (dadd.has_value() && dadd->defined()) {
      TORCH_CHECK(dadd->sizes() == x.sizes() && dadd->is_contiguous() && dadd->scalar_type() == x.scalar_type() &&
                      aligned16(*dadd), "rms_norm_bwd: dadd must match x");
      da = (const scalar_t*)dadd->data_ptr();
    }
    TB_CH_SWITCH(chn, launch_bwd<scalar_t, CH>(dyc, xc, wc, rstd, dx, need_dw ? part.data_ptr<float>() : nullptr,
                                               blocks, da));
  });
  check_launch("rms_norm_bwd");
  if (need_dw) {
    colsum_par_kernel<<<(D + 31) / 32, dim3(32, 16), 0, stream()>>>(part.data_ptr<float>(), dw.data_ptr<float>(),
                                                                  blocks, D);
    check_launch("rms_norm_bwd colsum");
  }
  return {dx, dw};
}

}  // namespace tb
