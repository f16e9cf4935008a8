// Causal depthwise conv1d + bias + SiLU (+ row L2-normalisation), forward and
// backward.  Forward: one warp per (b, t) row reads the K input rows it needs
// (neighbouring warps share them through L1/L2) and writes the finished row.
// Backward: kernel A recomputes the forward for a row and writes dc, the
// gradient at the conv output (fp32); kernel B (column slabs x row groups)
// forms dx by the transposed convolution of dc and accumulates dw/db partials
// in registers, reduced in a fixed order (deterministic).
#include "common.cuh"

namespace tb {

constexpr float kL2Eps = 1e-12f;  // F.normalize default eps

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&o)[4]) {
  if constexpr (sizeof(T) == 4) {
    float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  } else {
    union { uint2 r; T h[4]; } u;
    u.r = *reinterpret_cast<const uint2*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = to_f<T>(u.h[i]);
  }
}
template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&o)[4]) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  } else {
    union { uint2 r; T h[4]; } u;
#pragma unroll
    for (int i = 0; i < 4; ++i) u.h[i] = from_f<T>(o[i]);
    *reinterpret_cast<uint2*>(p) = u.r;
  }
}

// wt: [K, D] fp32 (transposed weights) or null; bias: [D] fp32 or null.
template <typename T, int CH>
__global__ void __launch_bounds__(256) conv_fwd_kernel(const T* __restrict__ x, int64_t sb, int64_t st,
                                                       const float* __restrict__ wt, const float* __restrict__ bias,
                                                       T* __restrict__ y, int B, int Tn, int D, int K, bool normalize) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * Tn;
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const int b = (int)(r / Tn), t = (int)(r % Tn);
    const T* xb = x + (int64_t)b * sb;
    float v[CH][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) {
        float acc[4];
        if (wt != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] = bias ? bias[col + i] : 0.f;
          for (int j = 0; j < K; ++j) {
            const int tt = t - K + 1 + j;
            if (tt < 0) continue;
            float xv[4];
            load4<T>(xb + (int64_t)tt * st + col, xv);
            const float4 ww = *reinterpret_cast<const float4*>(wt + (int64_t)j * D + col);
            acc[0] += ww.x * xv[0]; acc[1] += ww.y * xv[1]; acc[2] += ww.z * xv[2]; acc[3] += ww.w * xv[3];
          }
        } else {
          load4<T>(xb + (int64_t)t * st + col, acc);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[c][i] = silu_(acc[i]);
          ss += v[c][i] * v[c][i];
        }
      }
    }
    float inv = 1.f;
    if (normalize) inv = 1.f / fmaxf(sqrtf(warp_sum(ss)), kL2Eps);
    T* yr = y + r * D;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[c][i] *= inv;
        store4<T>(yr + col, v[c]);
      }
    }
  }
}

// Kernel A: dc = d(loss)/d(conv output), fp32 [B*T, D]; when there is no conv
// it writes dx (type T) directly.
template <typename T, int CH>
__global__ void __launch_bounds__(256) conv_bwd_a_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                         int64_t sb, int64_t st, const float* __restrict__ wt,
                                                         const float* __restrict__ bias, float* __restrict__ dc,
                                                         T* __restrict__ dx_direct, int B, int Tn, int D, int K,
                                                         bool normalize) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * Tn;
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = warp0; r < rows; r += nwarps) {
    const int b = (int)(r / Tn), t = (int)(r % Tn);
    const T* xb = x + (int64_t)b * sb;
    float pre[CH][4], s[CH][4], g[CH][4];
    float ss = 0.f, sd = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) {
        if (wt != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) pre[c][i] = bias ? bias[col + i] : 0.f;
          for (int j = 0; j < K; ++j) {
            const int tt = t - K + 1 + j;
            if (tt < 0) continue;
            float xv[4];
            load4<T>(xb + (int64_t)tt * st + col, xv);
            const float4 ww = *reinterpret_cast<const float4*>(wt + (int64_t)j * D + col);
            pre[c][0] += ww.x * xv[0]; pre[c][1] += ww.y * xv[1]; pre[c][2] += ww.z * xv[2]; pre[c][3] += ww.w * xv[3];
          }
        } else {
          load4<T>(xb + (int64_t)t * st + col, pre[c]);
        }
        load4<T>(dy + r * D + col, g[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          s[c][i] = silu_(pre[c][i]);
          ss += s[c][i] * s[c][i];
        }
      }
    }
    if (normalize) {
      const float nrm = sqrtf(warp_sum(ss));
      const float den = fmaxf(nrm, kL2Eps);
      // y = s / den; for nrm > eps: ds = (g - y (y.g)) / den ; else ds = g / eps
      if (nrm > kL2Eps) {
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          if (col < D)
#pragma unroll
            for (int i = 0; i < 4; ++i) sd += s[c][i] * g[c][i];
        }
        sd = warp_sum(sd) / (den * den);
      }
#pragma unroll
      for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) g[c][i] = (g[c][i] - s[c][i] * sd) / den;
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) {
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = g[c][i] * silu_grad_(pre[c][i]);
        if (dc != nullptr) {
          *reinterpret_cast<float4*>(dc + r * D + col) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          store4<T>(dx_direct + (int64_t)b * Tn * D + (int64_t)t * D + col, o);
        }
      }
    }
  }
}

// Kernel B: grid (D/128 column slabs, row groups); block 8 warps.
template <typename T>
__global__ void __launch_bounds__(256) conv_bwd_b_kernel(const float* __restrict__ dc, const T* __restrict__ x,
                                                         int64_t sb, int64_t st, const float* __restrict__ wt,
                                                         T* __restrict__ dx, float* __restrict__ part, int B, int Tn,
                                                         int D, int K) {
  constexpr int KMAX = 8;
  __shared__ float red[8][KMAX + 1][128];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int col = blockIdx.x * 128 + lane * 4;
  const bool active = col < D;
  float aw[KMAX][4], ab[4];
#pragma unroll
  for (int j = 0; j < KMAX; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) aw[j][i] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ab[i] = 0.f;
  const int64_t rows = (int64_t)B * Tn;
  if (active) {
    for (int64_t r = (int64_t)blockIdx.y * 8 + wid; r < rows; r += (int64_t)gridDim.y * 8) {
      const int b = (int)(r / Tn), t = (int)(r % Tn);
      const float4 g4 = *reinterpret_cast<const float4*>(dc + r * D + col);
      const float g[4] = {g4.x, g4.y, g4.z, g4.w};
      ab[0] += g[0]; ab[1] += g[1]; ab[2] += g[2]; ab[3] += g[3];
      const T* xb = x + (int64_t)b * sb;
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        if (j >= K) break;
        // dw[d, j] += dc[t, d] * x[t - K + 1 + j, d]
        const int tt = t - K + 1 + j;
        if (tt >= 0) {
          float xv[4];
          load4<T>(xb + (int64_t)tt * st + col, xv);
#pragma unroll
          for (int i = 0; i < 4; ++i) aw[j][i] += g[i] * xv[i];
        }
        // dx[t, d] += w[d, j] * dc[t + K - 1 - j, d]
        const int tf = t + K - 1 - j;
        if (tf < Tn) {
          const float4 d4 = *reinterpret_cast<const float4*>(dc + (r + (K - 1 - j)) * D + col);
          const float4 ww = *reinterpret_cast<const float4*>(wt + (int64_t)j * D + col);
          o[0] += ww.x * d4.x; o[1] += ww.y * d4.y; o[2] += ww.z * d4.z; o[3] += ww.w * d4.w;
        }
      }
      store4<T>(dx + r * D + col, o);
    }
  }
  if (part == nullptr) return;
#pragma unroll
  for (int j = 0; j < KMAX; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[wid][j][lane * 4 + i] = aw[j][i];
#pragma unroll
  for (int i = 0; i < 4; ++i) red[wid][KMAX][lane * 4 + i] = ab[i];
  __syncthreads();
  // part layout: [gridDim.y][K + 1][D]  (rows 0..K-1 = dw taps, row K = db)
  for (int e = threadIdx.x; e < (K + 1) * 128; e += blockDim.x) {
    const int j = e / 128, cc = e % 128;
    const int gcol = blockIdx.x * 128 + cc;
    if (gcol >= D) continue;
    const int src = (j == K) ? KMAX : j;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][src][cc];
    part[((int64_t)blockIdx.y * (K + 1) + j) * D + gcol] = s;
  }
}

__global__ void colsum_kernel2(const float* __restrict__ part, float* __restrict__ out, int G, int64_t N) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  float s = 0.f;
  for (int g = 0; g < G; ++g) s += part[(int64_t)g * N + i];
  out[i] = s;
}

#define TB_CH4_SWITCH(CHN, ...)                              \
  switch (CHN) {                                             \
    case 1: { constexpr int CH = 1; __VA_ARGS__; break; }    \
    case 2: { constexpr int CH = 2; __VA_ARGS__; break; }    \
    case 3: { constexpr int CH = 3; __VA_ARGS__; break; }    \
    case 4: { constexpr int CH = 4; __VA_ARGS__; break; }    \
    case 5: case 6: { constexpr int CH = 6; __VA_ARGS__; break; } \
    case 7: case 8: { constexpr int CH = 8; __VA_ARGS__; break; } \
    case 9: case 10: case 11: case 12: { constexpr int CH = 12; __VA_ARGS__; break; } \
    default: { constexpr int CH = 16; __VA_ARGS__; break; }  \
  }

static at::Tensor conv_wt(const c10::optional<at::Tensor>& w, int D) {
  if (!w.has_value() || !w->defined()) return at::Tensor();
  // [D, 1, K] -> [K, D] fp32
  return w->reshape({D, -1}).t().contiguous().to(at::kFloat);
}

at::Tensor conv_silu_norm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w,
                              const c10::optional<at::Tensor>& b, bool normalize) {
  TB_CHECK_CUDA(x);
  TB_CHECK_LASTDIM(x);
  TORCH_CHECK(x.dim() == 3, "conv_silu_norm: x must be [B, T, D]");
  const at::cuda::CUDAGuard g(x.device());
  const int B = x.size(0), Tn = x.size(1), D = x.size(2);
  TORCH_CHECK(D % 4 == 0 && x.stride(1) % 4 == 0 && x.stride(0) % 4 == 0, "conv_silu_norm: D and strides must be multiples of 4");
  TORCH_CHECK(((uintptr_t)x.data_ptr() % (4 * x.element_size())) == 0, "conv_silu_norm: x must be aligned to 4 elements");
  at::Tensor wt = conv_wt(w, D);
  const int K = wt.defined() ? wt.size(0) : 0;
  TORCH_CHECK(K <= 8, "conv kernel size must be <= 8");
  at::Tensor bias = (b.has_value() && b->defined()) ? b->to(at::kFloat).contiguous() : at::Tensor();
  at::Tensor y = at::empty({B, Tn, D}, x.options());
  const int64_t rows = (int64_t)B * Tn;
  if (rows == 0) return y;
  const int chn = (D + 127) / 128;
  TORCH_CHECK(chn <= 16, "conv_silu_norm: D too large");
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 8));
  TB_DISPATCH_FLOAT(x.scalar_type(), "conv_silu_norm_fwd", [&] {
    TB_CH4_SWITCH(chn, conv_fwd_kernel<scalar_t, CH><<<blocks, 256, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1), wt.defined() ? wt.data_ptr<float>() : nullptr,
        bias.defined() ? bias.data_ptr<float>() : nullptr, (scalar_t*)y.data_ptr(), B, Tn, D, K, normalize));
  });
  check_launch("conv_silu_norm_fwd");
  return y;
}

std::vector<at::Tensor> conv_silu_norm_bwd(const at::Tensor& dy, const at::Tensor& x,
                                           const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                                           bool normalize, bool need_wgrad) {
  TB_CHECK_CUDA(x);
  const at::cuda::CUDAGuard g(x.device());
  const int B = x.size(0), Tn = x.size(1), D = x.size(2);
  at::Tensor dyc = contig16(dy);
  TORCH_CHECK(x.stride(2) == 1 && x.stride(1) % 4 == 0 && x.stride(0) % 4 == 0 && D % 4 == 0 &&
              ((uintptr_t)x.data_ptr() % (4 * x.element_size())) == 0, "conv_silu_norm_bwd: x layout");
  at::Tensor wt = conv_wt(w, D);
  const int K = wt.defined() ? wt.size(0) : 0;
  at::Tensor bias = (b.has_value() && b->defined()) ? b->to(at::kFloat).contiguous() : at::Tensor();
  at::Tensor dx = at::empty({B, Tn, D}, x.options());
  at::Tensor dw = at::empty({0}, x.options().dtype(at::kFloat)), db = at::empty({0}, x.options().dtype(at::kFloat));
  const int64_t rows = (int64_t)B * Tn;
  if (rows == 0) return {dx.zero_(), dw, db};
  const int chn = (D + 127) / 128;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 8));
  at::Tensor dc = wt.defined() ? at::empty({B, Tn, D}, x.options().dtype(at::kFloat)) : at::Tensor();
  TB_DISPATCH_FLOAT(x.scalar_type(), "conv_silu_norm_bwd", [&] {
    TB_CH4_SWITCH(chn, conv_bwd_a_kernel<scalar_t, CH><<<blocks, 256, 0, stream()>>>(
        (const scalar_t*)dyc.data_ptr(), (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1),
        wt.defined() ? wt.data_ptr<float>() : nullptr, bias.defined() ? bias.data_ptr<float>() : nullptr,
        dc.defined() ? dc.data_ptr<float>() : nullptr, (scalar_t*)dx.data_ptr(), B, Tn, D, K, normalize));
    check_launch("conv_silu_norm_bwd_a");
    if (wt.defined()) {
      const int gy = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms() * 4 / ((D + 127) / 128) + 1));
      at::Tensor part = need_wgrad ? at::empty({gy, K + 1, D}, x.options().dtype(at::kFloat)) : at::Tensor();
      dim3 grid((D + 127) / 128, gy);
      conv_bwd_b_kernel<scalar_t><<<grid, 256, 0, stream()>>>(
          dc.data_ptr<float>(), (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1), wt.data_ptr<float>(),
          (scalar_t*)dx.data_ptr(), need_wgrad ? part.data_ptr<float>() : nullptr, B, Tn, D, K);
      check_launch("conv_silu_norm_bwd_b");
      if (need_wgrad) {
        at::Tensor red = at::empty({K + 1, D}, x.options().dtype(at::kFloat));
        const int64_t N = (int64_t)(K + 1) * D;
        colsum_kernel2<<<(N + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), red.data_ptr<float>(), gy, N);
        check_launch("conv_silu_norm_bwd colsum");
        dw = red.narrow(0, 0, K).t().contiguous();  // [D, K]
        db = red[K].contiguous();
      }
    }
  });
  return {dx, dw, db};
}

}  // namespace tb
