// AdamW over flat parameter buffers, with the global-norm gradient clip
// applied inside the update (the clip coefficient is computed on the device;
// nothing is read back to the host).
//
// Buffers: master (fp32), exp_avg / exp_avg_sq (fp32), grads (bf16 or fp32),
// optional low-precision parameter copy written from the updated master.
// `segs` is a device int64 [nseg, 2] table of (offset, length) ranges that
// received a gradient this step; parameters outside it are left untouched,
// matching torch.optim.AdamW's skip of parameters whose .grad is None.
// Offsets and lengths are multiples of 8 (parameters are padded to 64
// elements), so every thread moves 8 elements with 16/32-byte accesses.
#include "common.cuh"

namespace tb {

constexpr int kChunk = 1 << 14;  // elements per work item

// work items: (segment, chunk within segment) enumerated by a prefix table
// on the device: item_start[s] = first item of segment s.
__device__ __forceinline__ int find_seg(const int64_t* __restrict__ item_start, int nseg, int64_t item) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (item_start[mid] <= item) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// 8 consecutive elements as fp32 (16-byte bf16 or 2 x 16-byte fp32 accesses)
template <typename T>
__device__ __forceinline__ void ld8(const T* __restrict__ p, float (&o)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    load16<T>(p, o);
  }
}
template <typename T>
__device__ __forceinline__ void st8(T* __restrict__ p, const float (&o)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(o[4], o[5], o[6], o[7]);
  } else {
    store16<T>(p, o);
  }
}

template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ g, const int64_t* __restrict__ segs,
                             const int64_t* __restrict__ item_start, int nseg, int64_t nitems, float scale,
                             float* __restrict__ part) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int s = find_seg(item_start, nseg, it);
    const int64_t off = segs[2 * s], len = segs[2 * s + 1];
    const int64_t c0 = (it - item_start[s]) * kChunk;
    const int64_t c1 = min(len, c0 + kChunk);
    for (int64_t i = c0 + threadIdx.x * 8; i < c1; i += blockDim.x * 8) {
      float x[8];
      ld8<G>(g + off + i, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += (x[k] * scale) * (x[k] * scale);
    }
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

// out[0] = total norm, out[1] = clip coefficient (1 when max_norm <= 0)
__global__ void clip_coef_kernel(const float* __restrict__ part, int n, float max_norm, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += part[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) {
    const float nrm = sqrtf(s);
    out[0] = nrm;
    out[1] = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
  }
}

template <typename G, typename P>
__global__ void adamw_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                             const G* __restrict__ g, P* __restrict__ pout, const int64_t* __restrict__ segs,
                             const int64_t* __restrict__ item_start, int nseg, int64_t nitems,
                             const float* __restrict__ clip, float gscale, float lr, float b1, float b2, float eps,
                             float wd, float bc1, float bc2_sqrt, const float* __restrict__ hyper) {
  if (hyper) {  // step-dependent values from the device (CUDA-graph replay)
    lr = hyper[1];
    bc1 = hyper[2];
    bc2_sqrt = hyper[3];
  }
  const float cg = gscale * (clip ? clip[1] : 1.f);
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  for (int64_t it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int s = find_seg(item_start, nseg, it);
    const int64_t off = segs[2 * s], len = segs[2 * s + 1];
    const int64_t c0 = (it - item_start[s]) * kChunk;
    const int64_t c1 = min(len, c0 + kChunk);
    for (int64_t i = off + c0 + threadIdx.x * 8; i < off + c1; i += blockDim.x * 8) {
      float g8[8], p8[8], m8[8], v8[8];
      ld8<G>(g + i, g8);
      ld8<float>(master + i, p8);
      ld8<float>(m + i, m8);
      ld8<float>(v + i, v8);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gr = g8[k] * cg;
        m8[k] = b1 * m8[k] + (1.f - b1) * gr;
        v8[k] = b2 * v8[k] + (1.f - b2) * gr * gr;
        p8[k] = p8[k] * decay - step * m8[k] / (sqrtf(v8[k]) / bc2_sqrt + eps);
      }
      st8<float>(m + i, m8);
      st8<float>(v + i, v8);
      st8<float>(master + i, p8);
      if (pout) st8<P>(pout + i, p8);
    }
  }
}

// hyper = [step, lr, 1 - b1^step, sqrt(1 - b2^step)] (fp32, device): advance
// the step and recompute the rest, with the learning-rate multiplier of a
// linear warm-up then cosine decay to min_ratio (applied to step - 1, as a
// scheduler stepped after each update does), or 1 without a schedule.
__global__ void adamw_hyper_kernel(float* __restrict__ hyper, float base_lr, float b1, float b2, int warmup,
                                   int total, float min_ratio, int use_schedule) {
  const float step = hyper[0] + 1.f;
  hyper[0] = step;
  float mult = 1.f;
  if (use_schedule) {
    const float k = step - 1.f;
    if (k < (float)warmup) {
      mult = k / (float)max(1, warmup);
    } else {
      const float progress = (k - (float)warmup) / (float)max(1, total - warmup);
      mult = fmaxf(min_ratio, 0.5f * (1.f + cosf(3.14159265358979f * progress)));
    }
  }
  hyper[1] = base_lr * mult;
  hyper[2] = 1.f - powf(b1, step);
  hyper[3] = sqrtf(1.f - powf(b2, step));
}

void adamw_hyper_step(at::Tensor& hyper, double base_lr, double beta1, double beta2, int64_t warmup, int64_t total,
                      double min_ratio, bool use_schedule) {
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.numel() == 4, "adamw_hyper: float[4]");
  const at::cuda::CUDAGuard guard(hyper.device());
  adamw_hyper_kernel<<<1, 1, 0, stream()>>>(hyper.data_ptr<float>(), (float)base_lr, (float)beta1, (float)beta2,
                                            (int)warmup, (int)total, (float)min_ratio, use_schedule ? 1 : 0);
  check_launch("adamw_hyper_step");
}

// `tab` (device int64): [off0, len0, off1, len1, ..., item_start0, item_start1, ...]
// with item_start[s] = first kChunk-sized work item of segment s; built once
// on the host by the Python optimizer and cached on the device.
// Returns float[2] on device: (grad norm, clip coef).  `gscale` multiplies
// the raw grads first (e.g. 1/world_size for averaged data-parallel grads).
at::Tensor grad_norm_clip(const at::Tensor& grads, const at::Tensor& tab, int64_t nseg, int64_t items, double gscale,
                          double max_norm) {
  const at::cuda::CUDAGuard guard(grads.device());
  at::Tensor out = at::zeros({2}, grads.options().dtype(at::kFloat));
  if (nseg == 0) return out;
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.numel() == 3 * nseg, "grad_norm: bad table");
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms() * 4));
  at::Tensor part = at::empty({blocks}, grads.options().dtype(at::kFloat));
  const int64_t* segs = tab.data_ptr<int64_t>();
  const int64_t* istart = segs + 2 * nseg;
  if (grads.scalar_type() == at::kBFloat16) {
    sumsq_kernel<__nv_bfloat16><<<blocks, 512, 0, stream()>>>((const __nv_bfloat16*)grads.data_ptr(), segs, istart,
                                                             nseg, items, (float)gscale, part.data_ptr<float>());
  } else {
    TORCH_CHECK(grads.scalar_type() == at::kFloat, "grad_norm: bf16 or fp32 grads");
    sumsq_kernel<float><<<blocks, 512, 0, stream()>>>(grads.data_ptr<float>(), segs, istart, nseg, items,
                                                      (float)gscale, part.data_ptr<float>());
  }
  clip_coef_kernel<<<1, 1024, 0, stream()>>>(part.data_ptr<float>(), blocks, (float)max_norm, out.data_ptr<float>());
  check_launch("grad_norm_clip");
  return out;
}

void adamw_step(at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq, const at::Tensor& grads,
                const c10::optional<at::Tensor>& params_out, const at::Tensor& tab, int64_t nseg, int64_t items,
                const c10::optional<at::Tensor>& clip, double gscale, double lr, double beta1, double beta2,
                double eps, double wd, int64_t step, const c10::optional<at::Tensor>& hyper) {
  const at::cuda::CUDAGuard guard(master.device());
  TORCH_CHECK(master.scalar_type() == at::kFloat && exp_avg.scalar_type() == at::kFloat &&
                  exp_avg_sq.scalar_type() == at::kFloat, "adamw: fp32 master/state");
  TORCH_CHECK(master.numel() == grads.numel() && master.is_contiguous() && grads.is_contiguous(), "adamw: sizes");
  if (nseg == 0) return;
  TORCH_CHECK(tab.is_cuda() && tab.scalar_type() == at::kLong && tab.numel() == 3 * nseg, "adamw: bad table");
  const int64_t* segs = tab.data_ptr<int64_t>();
  const int64_t* istart = segs + 2 * nseg;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms() * 8));
  const float bc1 = 1.f - (float)std::pow(beta1, (double)step);
  const float bc2s = std::sqrt(1.f - (float)std::pow(beta2, (double)step));
  const float* cl = (clip.has_value() && clip->defined()) ? clip->data_ptr<float>() : nullptr;
  const bool has_out = params_out.has_value() && params_out->defined();
  auto launch = [&](auto gtag, auto ptag) {
    using G = decltype(gtag);
    using P = decltype(ptag);
    adamw_kernel<G, P><<<blocks, 512, 0, stream()>>>(
        master.data_ptr<float>(), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), (const G*)grads.data_ptr(),
        has_out ? (P*)params_out->data_ptr() : nullptr, segs, istart, nseg, items, cl, (float)gscale, (float)lr,
        (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2s,
        (hyper.has_value() && hyper->defined()) ? hyper->data_ptr<float>() : nullptr);
  };
  const bool gb = grads.scalar_type() == at::kBFloat16;
  const bool pb = !has_out || params_out->scalar_type() == at::kBFloat16;
  if (has_out) TORCH_CHECK(params_out->numel() == master.numel(), "adamw: params_out size");
  if (gb && pb) launch(__nv_bfloat16{}, __nv_bfloat16{});
  else if (gb && !pb) launch(__nv_bfloat16{}, float{});
  else if (!gb && pb) launch(float{}, __nv_bfloat16{});
  else launch(float{}, float{});
  check_launch("adamw_step");
}

}  // namespace tb
