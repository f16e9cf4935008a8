// Weight-only int8: per-output-row symmetric quantisation and the decode GEMM.
//
// W [N, K] bf16 -> q [N, K] int8 and s [N] fp32 with W ~ s[n] * q[n, k]
// (s[n] = max_k |W[n, k]| / 127, round to nearest).
//
// int8_gemm_small: y[m, n] = s[n] * sum_k x[m, k] q[n, k] for M <= 16 rows of
// bf16 activations (token-by-token decoding, small batches).  The product is
// bound by the weight bytes, so the weights are read once, 16 int8 per lane
// per load (each warp walks 2 rows, lanes striding K), dequantised in
// registers and multiplied with the activations (kept in shared memory for
// the whole K); fp32 accumulation, lane partials summed with shuffles.
// Larger M dequantises into a bf16 buffer and runs the tensor-core GEMM
// (host side).
#include "common.cuh"

namespace tb {
namespace quant {

constexpr int ROWS_PER_WARP = 2;
constexpr int WARPS = 8;

__global__ void quantize_rows_kernel(const __nv_bfloat16* __restrict__ w, int8_t* __restrict__ q,
                                     float* __restrict__ s, int N, int K) {
  const int row = blockIdx.x;
  if (row >= N) return;
  const __nv_bfloat16* wr = w + (int64_t)row * K;
  __shared__ float red[32];
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(__bfloat162float(wr[k])));
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float scale = red[0] > 0.f ? red[0] / 127.f : 1.f;
  if (threadIdx.x == 0) s[row] = scale;
  const float inv = 1.f / scale;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = rintf(__bfloat162float(wr[k]) * inv);
    q[(int64_t)row * K + k] = (int8_t)fmaxf(-127.f, fminf(127.f, v));
  }
}

__global__ void dequantize_kernel(const int8_t* __restrict__ q, const float* __restrict__ s,
                                  __nv_bfloat16* __restrict__ w, int64_t N, int K) {
  const int64_t n16 = N * K / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 16;
    const float sc = s[e / K];
    const int4 raw = reinterpret_cast<const int4*>(q)[i];
    const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
    Vec16<__nv_bfloat16> o0, o1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o0.v[j] = __float2bfloat16_rn(sc * (float)b[j]);
      o1.v[j] = __float2bfloat16_rn(sc * (float)b[8 + j]);
    }
    reinterpret_cast<uint4*>(w + e)[0] = o0.raw;
    reinterpret_cast<uint4*>(w + e)[1] = o1.raw;
  }
}

// grid: ceil(N / (WARPS * ROWS_PER_WARP)); block: 32 * WARPS; dynamic smem: M * K bf16
template <int M>
__global__ void __launch_bounds__(32 * WARPS) int8_gemm_small_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                    const int8_t* __restrict__ q,
                                                                    const float* __restrict__ s,
                                                                    __nv_bfloat16* __restrict__ y, int64_t ldy, int N,
                                                                    int K) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  // activations into shared memory (16-byte pieces)
  const int pieces = M * K / 8;
  for (int i = threadIdx.x; i < pieces; i += blockDim.x) {
    const int m = i / (K / 8), c = i - m * (K / 8);
    reinterpret_cast<uint4*>(xs)[i] = *reinterpret_cast<const uint4*>(x + (int64_t)m * ldx + c * 8);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * WARPS + warp) * ROWS_PER_WARP;
  if (row0 >= N) return;
  float acc[ROWS_PER_WARP][M];
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  for (int k0 = lane * 16; k0 < K; k0 += 32 * 16) {
    int4 raw[ROWS_PER_WARP];
#pragma unroll
    for (int r = 0; r < ROWS_PER_WARP; ++r)
      raw[r] = row0 + r < N ? __ldg(reinterpret_cast<const int4*>(q + (int64_t)(row0 + r) * K + k0))
                            : make_int4(0, 0, 0, 0);
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float xv[16];
      const uint4 a = *reinterpret_cast<const uint4*>(xs + m * K + k0);
      const uint4 b = *reinterpret_cast<const uint4*>(xs + m * K + k0 + 8);
      const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xv[j] = __bfloat162float(ap[j]);
        xv[8 + j] = __bfloat162float(bp[j]);
      }
#pragma unroll
      for (int r = 0; r < ROWS_PER_WARP; ++r) {
        const int8_t* qb = reinterpret_cast<const int8_t*>(&raw[r]);
        float t = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) t = fmaf(xv[j], (float)qb[j], t);
        acc[r][m] += t;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    const int n = row0 + r;
    const float sc = n < N ? s[n] : 0.f;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && n < N) y[(int64_t)m * ldy + n] = __float2bfloat16_rn(v * sc);
    }
  }
}

}  // namespace quant

std::vector<at::Tensor> quantize_int8_rows(const at::Tensor& w) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.is_contiguous(),
              "quantize_int8_rows: contiguous bf16 [N, K] CUDA tensor");
  const at::cuda::CUDAGuard g(w.device());
  const int N = (int)w.size(0), K = (int)w.size(1);
  at::Tensor q = at::empty({N, K}, w.options().dtype(at::kChar));
  at::Tensor s = at::empty({N}, w.options().dtype(at::kFloat));
  if (N > 0)
    quant::quantize_rows_kernel<<<N, 256, 0, stream()>>>((const __nv_bfloat16*)w.data_ptr(), q.data_ptr<int8_t>(),
                                                         s.data_ptr<float>(), N, K);
  check_launch("quantize_int8_rows");
  return {q, s};
}

at::Tensor dequantize_int8_rows(const at::Tensor& q, const at::Tensor& s) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous() &&
                  q.size(1) % 16 == 0 && s.scalar_type() == at::kFloat && s.numel() == q.size(0),
              "dequantize_int8_rows: q int8 [N, K] (K % 16 == 0), s fp32 [N]");
  const at::cuda::CUDAGuard g(q.device());
  at::Tensor w = at::empty(q.sizes(), q.options().dtype(at::kBFloat16));
  const int64_t n16 = q.numel() / 16;
  if (n16 > 0) {
    const int blocks = (int)std::min<int64_t>((n16 + 255) / 256, (int64_t)num_sms() * 8);
    quant::dequantize_kernel<<<blocks, 256, 0, stream()>>>(q.data_ptr<int8_t>(), s.data_ptr<float>(),
                                                           (__nv_bfloat16*)w.data_ptr(), q.size(0), (int)q.size(1));
  }
  check_launch("dequantize_int8_rows");
  return w;
}

// y [M, N] bf16 = x [M, K] bf16 . (s * q)^T for M <= 16
at::Tensor int8_gemm_small(const at::Tensor& x, const at::Tensor& q, const at::Tensor& s) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "int8_gemm_small: x bf16 [M, K] with contiguous rows");
  TORCH_CHECK(q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous() && q.size(1) == x.size(1) &&
                  s.scalar_type() == at::kFloat && s.numel() == q.size(0),
              "int8_gemm_small: q int8 [N, K], s fp32 [N]");
  const int M = (int)x.size(0), N = (int)q.size(0), K = (int)x.size(1);
  TORCH_CHECK(M >= 1 && M <= 16 && K % 16 == 0 && x.stride(0) % 8 == 0 && aligned16(x) && aligned16(q),
              "int8_gemm_small: 1 <= M <= 16, K % 16 == 0, 16-byte aligned rows");
  TORCH_CHECK((int64_t)M * K * 2 <= 200 * 1024, "int8_gemm_small: activations exceed shared memory");
  const at::cuda::CUDAGuard g(x.device());
  // the kernel is specialised for 1, 2, 4, 8 and 16 rows; other counts run padded with zero rows
  const int Mp = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
  at::Tensor xin = x;
  if (Mp != M) {
    xin = at::zeros({Mp, K}, x.options());
    xin.narrow(0, 0, M).copy_(x);
  }
  at::Tensor y = at::empty({Mp, N}, x.options());
  const int rows_per_block = quant::WARPS * quant::ROWS_PER_WARP;
  const dim3 grid((N + rows_per_block - 1) / rows_per_block);
  const size_t smem = (size_t)Mp * K * 2;
  const auto* xp = (const __nv_bfloat16*)xin.data_ptr();
  const int64_t ldx = xin.stride(0);
  auto* yp = (__nv_bfloat16*)y.data_ptr();
  auto launch = [&](auto kern) {
    if (smem > 48 * 1024)
      C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, 32 * quant::WARPS, smem, stream()>>>(xp, ldx, q.data_ptr<int8_t>(), s.data_ptr<float>(), yp, N, N,
                                                       K);
  };
  if (N > 0) {
    switch (Mp) {
      case 1: launch(quant::int8_gemm_small_kernel<1>); break;
      case 2: launch(quant::int8_gemm_small_kernel<2>); break;
      case 4: launch(quant::int8_gemm_small_kernel<4>); break;
      case 8: launch(quant::int8_gemm_small_kernel<8>); break;
      default: launch(quant::int8_gemm_small_kernel<16>); break;
    }
  }
  check_launch("int8_gemm_small");
  return Mp == M ? y : y.narrow(0, 0, M).contiguous();
}

}  // namespace tb
