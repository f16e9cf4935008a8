// Fused softmax cross-entropy over the vocabulary (mean over non-ignored rows).
// Forward: one block per row streams the logits once with an online
// max/sum-of-exp, writes the row's log-sum-exp and loss; a second kernel sums
// the row losses in a fixed order.  Backward recomputes softmax from the saved
// log-sum-exp and writes d(logits) = (softmax - onehot) * g / count, with g
// and count read from device memory (no host synchronisation).
#include "common.cuh"

namespace tb {

struct MaxSum {
  float m, s;
};
__device__ __forceinline__ MaxSum ms_combine(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

template <typename T>
__global__ void __launch_bounds__(256) ce_fwd_kernel(const T* __restrict__ logits, int64_t ls,
                                                     const int64_t* __restrict__ labels, float* __restrict__ lse_out,
                                                     float* __restrict__ row_loss, int V, int64_t ignore_index,
                                                     bool vec) {
  constexpr int VEC = Vec16<T>::N;
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ls;
  MaxSum acc{-INFINITY, 0.f};
  const int nvec = vec ? V / VEC : 0;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[VEC];
    load16<T>(lr + (int64_t)i * VEC, v);
    float m = v[0];
#pragma unroll
    for (int k = 1; k < VEC; ++k) m = fmaxf(m, v[k]);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VEC; ++k) s += __expf(v[k] - m);
    acc = ms_combine(acc, {m, s});
  }
  for (int i = nvec * VEC + threadIdx.x; i < V; i += blockDim.x) acc = ms_combine(acc, {to_f<T>(lr[i]), 1.f});
  // warp then block combine
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = ms_combine(acc, other);
  }
  __shared__ float sm[32], ss[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { sm[wid] = acc.m; ss[wid] = acc.s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    MaxSum t{sm[0], ss[0]};
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) t = ms_combine(t, {sm[k], ss[k]});
    const float lse = t.m + __logf(t.s);
    lse_out[row] = lse;
    const int64_t y = labels[row];
    row_loss[row] = (y == ignore_index || y < 0 || y >= V) ? 0.f : lse - to_f<T>(lr[y]);
  }
}

// out[0] = mean loss over valid rows, out[1] = number of valid rows (as float)
__global__ void ce_reduce_kernel(const float* __restrict__ row_loss, const int64_t* __restrict__ labels, int64_t N,
                                 int V, int64_t ignore_index, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f, c = 0.f;
  for (int64_t i = threadIdx.x; i < N; i += blockDim.x) {
    s += row_loss[i];
    const int64_t y = labels[i];
    c += (y == ignore_index || y < 0 || y >= V) ? 0.f : 1.f;
  }
  s = block_sum(s, red);
  c = block_sum(c, red);
  if (threadIdx.x == 0) {
    out[0] = c > 0.f ? s / c : NAN;
    out[1] = c;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ce_bwd_kernel(const T* __restrict__ logits, int64_t ls,
                                                     const int64_t* __restrict__ labels, const float* __restrict__ lse,
                                                     const float* __restrict__ stats, const float* __restrict__ gout,
                                                     T* __restrict__ dlogits, int V, int64_t ignore_index,
                                                     bool vec) {
  constexpr int VEC = Vec16<T>::N;
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ls;
  T* dr = dlogits + row * (int64_t)V;
  const int64_t y = labels[row];
  const bool valid = !(y == ignore_index || y < 0 || y >= V);
  const float scale = valid ? gout[0] / stats[1] : 0.f;
  const float l = lse[row];
  const int nvec = vec ? V / VEC : 0;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float v[VEC];
    load16<T>(lr + (int64_t)i * VEC, v);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const int col = i * VEC + k;
      v[k] = scale * (__expf(v[k] - l) - (col == y ? 1.f : 0.f));
    }
    store16<T>(dr + (int64_t)i * VEC, v);
  }
  for (int i = nvec * VEC + threadIdx.x; i < V; i += blockDim.x)
    dr[i] = from_f<T>(scale * (__expf(to_f<T>(lr[i]) - l) - (i == y ? 1.f : 0.f)));
}

// returns {stats[2] = (mean loss, count), lse[N]}
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& labels, int64_t ignore_index) {
  TB_CHECK_CUDA(logits);
  TB_CHECK_LASTDIM(logits);
  TORCH_CHECK(logits.dim() == 2 && labels.dim() == 1 && labels.size(0) == logits.size(0), "cross_entropy: shapes");
  const at::cuda::CUDAGuard g(logits.device());
  const int64_t N = logits.size(0);
  const int V = logits.size(1);
  at::Tensor lab = labels.to(at::kLong).contiguous();
  at::Tensor lse = at::empty({N}, logits.options().dtype(at::kFloat));
  at::Tensor rl = at::empty({N}, logits.options().dtype(at::kFloat));
  at::Tensor stats = at::empty({2}, logits.options().dtype(at::kFloat));
  TB_DISPATCH_FLOAT(logits.scalar_type(), "cross_entropy_fwd", [&] {
    constexpr int VEC = Vec16<scalar_t>::N;
    const bool vec = (logits.stride(0) % VEC == 0) && (V % VEC == 0) && ((uintptr_t)logits.data_ptr() % 16) == 0;
    if (N) ce_fwd_kernel<scalar_t><<<N, 256, 0, stream()>>>((const scalar_t*)logits.data_ptr(), logits.stride(0),
                                                            lab.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                                            rl.data_ptr<float>(), V, ignore_index, vec);
  });
  ce_reduce_kernel<<<1, 1024, 0, stream()>>>(rl.data_ptr<float>(), lab.data_ptr<int64_t>(), N, V, ignore_index,
                                              stats.data_ptr<float>());
  check_launch("cross_entropy_fwd");
  return {stats, lse};
}

at::Tensor cross_entropy_bwd(const at::Tensor& logits, const at::Tensor& labels, const at::Tensor& lse,
                             const at::Tensor& stats, const at::Tensor& gout, int64_t ignore_index) {
  const at::cuda::CUDAGuard g(logits.device());
  const int64_t N = logits.size(0);
  const int V = logits.size(1);
  at::Tensor lab = labels.to(at::kLong).contiguous();
  at::Tensor go = gout.to(at::kFloat).reshape({1}).contiguous();
  at::Tensor d = at::empty({N, V}, logits.options());
  TB_DISPATCH_FLOAT(logits.scalar_type(), "cross_entropy_bwd", [&] {
    constexpr int VEC = Vec16<scalar_t>::N;
    const bool vec = (logits.stride(0) % VEC == 0) && (V % VEC == 0) && ((uintptr_t)logits.data_ptr() % 16) == 0;
    if (N) ce_bwd_kernel<scalar_t><<<N, 256, 0, stream()>>>((const scalar_t*)logits.data_ptr(), logits.stride(0),
                                                            lab.data_ptr<int64_t>(), lse.data_ptr<float>(),
                                                            stats.data_ptr<float>(), go.data_ptr<float>(),
                                                            (scalar_t*)d.data_ptr(), V, ignore_index, vec);
  });
  check_launch("cross_entropy_bwd");
  return d;
}

}  // namespace tb
