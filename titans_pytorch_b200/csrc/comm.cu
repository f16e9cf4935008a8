// Data-parallel gradient reduction fused with clip + AdamW, over NVLink peer
// memory (one process per GPU; peers' buffers mapped with CUDA IPC).
//
// Buffers (every rank): flat bf16 gradient G_r and flat bf16 parameters P_r
// (peer-visible), a signal array and a norm-slot array (peer-visible), and,
// for its own shard [lo, lo + n) only, fp32 master weights and moments.
// One optimizer step:
//   barrier 0        every rank's backward has finished writing G
//   reduce_shard     g[i] = sum_r G_r[lo + i] (peer loads, fp32), kept in a
//                    local fp32 buffer, plus per-block partial sums of g^2
//   norm_publish     the shard's |g|^2 is written into slot[me] of every peer
//   barrier 1        all slots written
//   adamw_shard      clip coefficient from the slots; AdamW on the shard's
//                    active ranges; the new bf16 weights are stored straight
//                    into every peer's P (all-gather by peer stores)
//   barrier 2        every rank's P is complete before the next forward
// Barriers are epoch counters: rank s stores the epoch into sig[k][s] of every
// peer (release, system scope) and waits until its own sig[k][*] reach the
// epoch (acquire).  The epoch lives in a device word that the step's first
// barrier advances, so the step's launches are identical every step (CUDA-graph
// replay).  Every wait is bounded (~2^31 cycles); a timeout sets an
// error word and the kernel returns.  No multicast / NVLS is used.
#include "common.cuh"

namespace tb {
namespace comm {

constexpr int kChunk = 1 << 14;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// one block of `world` (>= 32 rounded) threads; epoch = *epoch_dev (+1, stored
// back, when `bump`)
__global__ void barrier_kernel(uint32_t* const* __restrict__ sig_ptrs, int slot, uint32_t* __restrict__ epoch_dev,
                               int bump, int world, int me, unsigned* __restrict__ err, long long budget) {
  const int t = threadIdx.x;
  __shared__ uint32_t ep;
  if (t == 0) {
    ep = *epoch_dev + (bump ? 1u : 0u);
    if (bump) *epoch_dev = ep;
  }
  __syncthreads();
  const uint32_t epoch = ep;
  __threadfence_system();  // everything this rank wrote before the barrier is visible system-wide
  if (t < world) st_release_sys(sig_ptrs[t] + slot * world + me, epoch);
  if (t < world) {
    const uint32_t* mine = sig_ptrs[me] + slot * world + t;
    const long long t0 = clock64();
    while (ld_acquire_sys(mine) < epoch) {
      if (clock64() - t0 > budget) {
        atomicCAS(err, 0u, 100u + (unsigned)slot);
        break;
      }
    }
  }
  __syncthreads();
}

// g = sum over ranks of G_r[lo + i], 8 elements per step; part[block] = sum g^2 * gscale^2
__global__ void reduce_shard_kernel(const __nv_bfloat16* const* __restrict__ grads, int64_t lo, int64_t n, int world,
                                    float* __restrict__ gsum, float gscale, float* __restrict__ part) {
  __shared__ float red[32];
  float acc = 0.f;
  const int64_t nv = n / 8;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r) {
      float x[8];
      load16<__nv_bfloat16>(grads[r] + lo + v * 8, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] += x[k];
    }
    float4* dst = reinterpret_cast<float4*>(gsum + v * 8);
    dst[0] = make_float4(s[0], s[1], s[2], s[3]);
    dst[1] = make_float4(s[4], s[5], s[6], s[7]);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += (s[k] * gscale) * (s[k] * gscale);
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

// Segment form (sharded-parameter layout): for segment s = (flat offset,
// shard offset, length), g[shard_off + i] = sum_r G_r[flat_off + i]; work
// items are kChunk-element pieces of the segments.
// `accumulate`: g[shard_off + i] += the sum (gradient accumulation over
// micro-batches whose gradients are reduced one by one); the partial norms
// are those of the accumulated values.
__global__ void reduce_segments_kernel(const __nv_bfloat16* const* __restrict__ grads,
                                       const int64_t* __restrict__ segs, const int64_t* __restrict__ item_start,
                                       int nseg, int64_t nitems, int world, float* __restrict__ gsum, float gscale,
                                       float* __restrict__ part, int accumulate);

// single block: slot[me] of every peer <- sum(part)
__global__ void norm_publish_kernel(const float* __restrict__ part, int nparts, float* const* __restrict__ slots,
                                    int world, int me) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
  s = block_sum(s, red);
  if (threadIdx.x < world) slots[threadIdx.x][me] = s;
  __threadfence_system();
}

__device__ __forceinline__ void load8f(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void store8f(float* p, const float (&o)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ int find_seg(const int64_t* __restrict__ item_start, int nseg, int64_t item) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (item_start[mid] <= item) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void reduce_segments_kernel(const __nv_bfloat16* const* __restrict__ grads,
                                       const int64_t* __restrict__ segs, const int64_t* __restrict__ item_start,
                                       int nseg, int64_t nitems, int world, float* __restrict__ gsum, float gscale,
                                       float* __restrict__ part, int accumulate) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int s = find_seg(item_start, nseg, it);
    const int64_t foff = segs[3 * s], soff = segs[3 * s + 1], len = segs[3 * s + 2];
    const int64_t c0 = (it - item_start[s]) * kChunk, c1 = min(len, c0 + kChunk);
    for (int64_t e = c0 + threadIdx.x * 8; e < c1; e += blockDim.x * 8) {
      float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < world; ++r) {
        float x[8];
        load16<__nv_bfloat16>(grads[r] + foff + e, x);
#pragma unroll
        for (int k = 0; k < 8; ++k) sum[k] += x[k];
      }
      float4* dst = reinterpret_cast<float4*>(gsum + soff + e);
      if (accumulate) {
        const float4 a = dst[0], b = dst[1];
        sum[0] += a.x; sum[1] += a.y; sum[2] += a.z; sum[3] += a.w;
        sum[4] += b.x; sum[5] += b.y; sum[6] += b.z; sum[7] += b.w;
      }
      dst[0] = make_float4(sum[0], sum[1], sum[2], sum[3]);
      dst[1] = make_float4(sum[4], sum[5], sum[6], sum[7]);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += (sum[k] * gscale) * (sum[k] * gscale);
    }
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) part[blockIdx.x] = acc;
}

// AdamW on the shard's active ranges (shard-relative offsets, multiples of 8),
// new bf16 weights stored into every rank's parameter buffer at lo + i.
// With `seg_aux` (sharded-parameter layout) segment s is stored at
// lo + i + seg_aux[2s] instead, into every rank's buffer when seg_aux[2s+1]
// is nonzero (replicated parameters) and into this rank's only otherwise
// (sharded parameters, gathered by the next forward).
__global__ void adamw_shard_kernel(const float* __restrict__ gsum, float* __restrict__ master, float* __restrict__ m,
                                   float* __restrict__ v, __nv_bfloat16* const* __restrict__ params, int64_t lo,
                                   int world, const int64_t* __restrict__ segs, const int64_t* __restrict__ item_start,
                                   int nseg, int64_t nitems, const float* __restrict__ norm_slots, float gscale,
                                   float max_norm, float lr, float b1, float b2, float eps, float wd, float bc1,
                                   float bc2_sqrt, float* __restrict__ norm_out, const float* __restrict__ hyper,
                                   const int64_t* __restrict__ seg_aux, int me) {
  if (hyper) {  // [step, lr, bc1, sqrt(bc2)] advanced on the device (CUDA-graph replay)
    lr = hyper[1];
    bc1 = hyper[2];
    bc2_sqrt = hyper[3];
  }
  float tot = 0.f;
  for (int r = 0; r < world; ++r) tot += norm_slots[r];
  const float nrm = sqrtf(tot);
  const float clip = max_norm > 0.f ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
  if (blockIdx.x == 0 && threadIdx.x == 0 && norm_out) norm_out[0] = nrm;
  const float cg = gscale * clip, step = lr / bc1, decay = 1.f - lr * wd;
  for (int64_t it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int s = find_seg(item_start, nseg, it);
    const int64_t off = segs[2 * s], len = segs[2 * s + 1];
    const int64_t c0 = (it - item_start[s]) * kChunk;
    const int64_t c1 = min(len, c0 + kChunk);
    const int64_t delta = seg_aux ? seg_aux[2 * s] : 0;
    const bool all_ranks = seg_aux ? seg_aux[2 * s + 1] != 0 : true;
    for (int64_t e = off + c0 + threadIdx.x * 8; e < off + c1; e += blockDim.x * 8) {
      float g8[8], p8[8], m8[8], v8[8], out[8];
      load8f(gsum + e, g8);
      load8f(master + e, p8);
      load8f(m + e, m8);
      load8f(v + e, v8);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gr = g8[k] * cg;
        const float p = p8[k] * decay;
        m8[k] = b1 * m8[k] + (1.f - b1) * gr;
        v8[k] = b2 * v8[k] + (1.f - b2) * gr * gr;
        out[k] = p - step * m8[k] / (sqrtf(v8[k]) / bc2_sqrt + eps);
      }
      store8f(master + e, out);
      store8f(m + e, m8);
      store8f(v + e, v8);
      Vec16<__nv_bfloat16> pk;
#pragma unroll
      for (int k = 0; k < 8; ++k) pk.v[k] = __float2bfloat16_rn(out[k]);
      if (all_ranks) {
        for (int r = 0; r < world; ++r) *reinterpret_cast<uint4*>(params[r] + lo + e + delta) = pk.raw;
      } else {
        *reinterpret_cast<uint4*>(params[me] + lo + e + delta) = pk.raw;
      }
    }
  }
  __threadfence_system();
}

}  // namespace comm

// ---------------------------------------------------------------- host API

static int64_t world_of(const at::Tensor& ptrs) { return ptrs.numel(); }

// Peer-shareable device buffer: cudaMalloc'd (not from PyTorch's caching
// allocator, so its IPC handle covers exactly this buffer).  Returns the
// buffer as a uint8 tensor (freed with cudaFree when the tensor dies) and its
// 64-byte IPC handle.
std::vector<at::Tensor> comm_alloc(int64_t nbytes, int64_t device) {
  const at::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)std::max<int64_t>(nbytes, 256)));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)std::max<int64_t>(nbytes, 256)));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto opts = at::TensorOptions().device(at::kCUDA, (c10::DeviceIndex)device).dtype(at::kByte);
  at::Tensor t = at::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
  at::Tensor ht = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(ht.data_ptr(), &h, sizeof(h));
  return {t, ht};
}

int64_t comm_ipc_open(const at::Tensor& handle, int64_t device) {
  const at::cuda::CUDAGuard g((c10::DeviceIndex)device);
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "comm_ipc_open: bad handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)(uintptr_t)p;
}

void comm_ipc_close(int64_t ptr) {
  if (ptr) C10_CUDA_CHECK(cudaIpcCloseMemHandle((void*)(uintptr_t)ptr));
}

// `budget`: clock cycles each wait may spin before it records 100 + slot in
// `err` and returns (default 2^31, about a second).
void comm_barrier(const at::Tensor& sig_ptrs, int64_t slot, at::Tensor& epoch, bool bump, int64_t world, int64_t me,
                  at::Tensor& err, int64_t budget) {
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() == 1, "comm_barrier: epoch word");
  TORCH_CHECK(budget > 0, "comm_barrier: budget must be positive");
  comm::barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, stream()>>>(
      reinterpret_cast<uint32_t* const*>(sig_ptrs.data_ptr<int64_t>()), (int)slot,
      reinterpret_cast<uint32_t*>(epoch.data_ptr<int>()), bump ? 1 : 0, (int)world, (int)me,
      (unsigned*)err.data_ptr<int>(), (long long)budget);
  check_launch("comm_barrier");
}

// Reduce-scatter of the bf16 gradient into gsum (fp32, shard length) and
// publication of the shard's squared norm into every peer's slot array.
void comm_reduce_shard(const at::Tensor& grad_ptrs, int64_t lo, int64_t n, at::Tensor& gsum, double gscale,
                       const at::Tensor& slot_ptrs, int64_t world, int64_t me) {
  TORCH_CHECK(n % 8 == 0 && lo % 8 == 0, "comm_reduce_shard: shard must be 8-element aligned");
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n / 8 + 255) / 256, (int64_t)num_sms() * 4));
  at::Tensor part = at::empty({blocks}, gsum.options());
  comm::reduce_shard_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16* const*>(grad_ptrs.data_ptr<int64_t>()), lo, n, (int)world,
      gsum.data_ptr<float>(), (float)gscale, part.data_ptr<float>());
  comm::norm_publish_kernel<<<1, 256, 0, stream()>>>(part.data_ptr<float>(), blocks,
                                                     reinterpret_cast<float* const*>(slot_ptrs.data_ptr<int64_t>()),
                                                     (int)world, (int)me);
  check_launch("comm_reduce_shard");
}

void comm_adamw_shard(const at::Tensor& gsum, at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                      const at::Tensor& param_ptrs, int64_t lo, int64_t world, const at::Tensor& tab, int64_t nseg,
                      int64_t items, const at::Tensor& norm_slots, double gscale, double max_norm, double lr,
                      double beta1, double beta2, double eps, double wd, int64_t step, at::Tensor& norm_out,
                      const c10::optional<at::Tensor>& hyper, const c10::optional<at::Tensor>& seg_aux, int64_t me) {
  if (nseg == 0) return;
  const int64_t* segs = tab.data_ptr<int64_t>();
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms() * 8));
  const float bc1 = 1.f - (float)std::pow(beta1, (double)step);
  const float bc2s = std::sqrt(1.f - (float)std::pow(beta2, (double)step));
  comm::adamw_shard_kernel<<<blocks, 256, 0, stream()>>>(
      gsum.data_ptr<float>(), master.data_ptr<float>(), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16* const*>(param_ptrs.data_ptr<int64_t>()), lo, (int)world, segs,
      segs + 2 * nseg, (int)nseg, items, norm_slots.data_ptr<float>(), (float)gscale, (float)max_norm, (float)lr,
      (float)beta1, (float)beta2, (float)eps, (float)wd, bc1, bc2s, norm_out.data_ptr<float>(),
      (hyper.has_value() && hyper->defined()) ? hyper->data_ptr<float>() : nullptr,
      (seg_aux.has_value() && seg_aux->defined()) ? seg_aux->data_ptr<int64_t>() : nullptr, (int)me);
  check_launch("comm_adamw_shard");
}

// Reduce-scatter in the sharded-parameter layout: `tab` = [nseg][3] (flat
// offset, shard offset, length; multiples of 8) followed by the segments'
// first work-item indices; then the shard's squared norm is published into
// every peer's slot array.
void comm_reduce_segments(const at::Tensor& grad_ptrs, const at::Tensor& tab, int64_t nseg, int64_t items,
                          at::Tensor& gsum, double gscale, const at::Tensor& slot_ptrs, int64_t world, int64_t me) {
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(items, num_sms() * 8));
  at::Tensor part = at::zeros({blocks}, gsum.options());
  if (nseg > 0) {
    const int64_t* segs = tab.data_ptr<int64_t>();
    comm::reduce_segments_kernel<<<blocks, 256, 0, stream()>>>(
        reinterpret_cast<const __nv_bfloat16* const*>(grad_ptrs.data_ptr<int64_t>()), segs, segs + 3 * nseg,
        (int)nseg, items, (int)world, gsum.data_ptr<float>(), (float)gscale, part.data_ptr<float>(), 0);
  }
  comm::norm_publish_kernel<<<1, 256, 0, stream()>>>(part.data_ptr<float>(), blocks,
                                                     reinterpret_cast<float* const*>(slot_ptrs.data_ptr<int64_t>()),
                                                     (int)world, (int)me);
  check_launch("comm_reduce_segments");
}

// Reduce-scatter of one unit's gradients without publishing the norm:
// block partials of the squared norm go to part[part_off, part_off + blocks)
// (`blocks` fixed by the caller, so every unit's slice of `part` is fixed and
// the launches are identical every step).  Runs on any stream (e.g. a
// communication stream while the backward of earlier layers continues).
void comm_reduce_into(const at::Tensor& grad_ptrs, const at::Tensor& tab, int64_t nseg, int64_t items,
                      at::Tensor& gsum, double gscale, at::Tensor& part, int64_t part_off, int64_t blocks,
                      bool accumulate) {
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == at::kFloat && part_off >= 0 && blocks > 0 &&
                  part_off + blocks <= part.numel(),
              "comm_reduce_into: partial-norm slice out of range");
  if (nseg == 0 || items == 0) {
    part.narrow(0, part_off, blocks).zero_();
    return;
  }
  const int64_t* segs = tab.data_ptr<int64_t>();
  comm::reduce_segments_kernel<<<(int)blocks, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16* const*>(grad_ptrs.data_ptr<int64_t>()), segs, segs + 3 * nseg,
      (int)nseg, items, (int)world_of(grad_ptrs), gsum.data_ptr<float>(), (float)gscale,
      part.data_ptr<float>() + part_off, accumulate ? 1 : 0);
  check_launch("comm_reduce_into");
}

// slot[me] of every peer <- sum(part[0, nparts))
void comm_norm_publish(const at::Tensor& part, int64_t nparts, const at::Tensor& slot_ptrs, int64_t world,
                       int64_t me) {
  TORCH_CHECK(nparts > 0 && nparts <= part.numel(), "comm_norm_publish: nparts");
  comm::norm_publish_kernel<<<1, 256, 0, stream()>>>(part.data_ptr<float>(), (int)nparts,
                                                     reinterpret_cast<float* const*>(slot_ptrs.data_ptr<int64_t>()),
                                                     (int)world, (int)me);
  check_launch("comm_norm_publish");
}

}  // namespace tb
