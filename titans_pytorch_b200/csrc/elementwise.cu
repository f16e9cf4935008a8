// Elementwise kernels: SwiGLU fwd/bwd, the memory-update epilogues
// (activation, scaled error, activation-gradient product, gated weight update)
// and the memory gates (sequence mean -> 3 gate GEMVs -> sigmoid means),
// which leave alpha/theta/eta in device memory (no host synchronisation).
#include "common.cuh"

namespace tb {

// ---------------------------------------------------------------- SwiGLU
// h = silu(gate) * up : [M, F]; gate row m at g + m * ldg, up row m at u + m * ldu
// (the stacked gu [M, 2F] = [gate | up] is g = gu, u = gu + F, ld = 2F)
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gp, int64_t ldg, const T* __restrict__ up, int64_t ldu,
                                  T* __restrict__ h, int64_t M, int F) {
  constexpr int V = Vec16<T>::N;
  const int64_t nvec = M * (F / V);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (F / V);
    const int c = (int)(i % (F / V)) * V;
    float g[V], u[V], o[V];
    load16<T>(gp + m * ldg + c, g);
    load16<T>(up + m * ldu + c, u);
#pragma unroll
    for (int k = 0; k < V; ++k) o[k] = silu_(g[k]) * u[k];
    store16<T>(h + m * F + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ gu, T* __restrict__ dgu,
                                  int64_t M, int F) {
  constexpr int V = Vec16<T>::N;
  const int64_t nvec = M * (F / V);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (F / V);
    const int c = (int)(i % (F / V)) * V;
    float g[V], u[V], d[V], dg[V], du[V];
    load16<T>(gu + m * 2 * F + c, g);
    load16<T>(gu + m * 2 * F + F + c, u);
    load16<T>(dh + m * F + c, d);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      dg[k] = d[k] * u[k] * silu_grad_(g[k]);
      du[k] = d[k] * silu_(g[k]);
    }
    store16<T>(dgu + m * 2 * F + c, dg);
    store16<T>(dgu + m * 2 * F + F + c, du);
  }
}

static int64_t ew_blocks(int64_t n) {
  return std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16));
}

at::Tensor swiglu_fwd(const at::Tensor& gu) {
  TB_CHECK_CUDA(gu);
  const at::cuda::CUDAGuard g(gu.device());
  at::Tensor x = contig16(gu);
  const int64_t M = x.size(0);
  const int F = x.size(1) / 2;
  at::Tensor h = at::empty({M, F}, x.options());
  TB_DISPATCH_FLOAT(x.scalar_type(), "swiglu_fwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(F % V == 0, "swiglu: F must be a multiple of ", V);
    const int64_t n = M * (F / V);
    const scalar_t* gp = (const scalar_t*)x.data_ptr();
    if (n) swiglu_fwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(gp, 2 * F, gp + F, 2 * F,
                                                                            (scalar_t*)h.data_ptr(), M, F);
  });
  check_launch("swiglu_fwd");
  return h;
}

// h = silu(g) * u for two same-shape tensors (any leading shape, flattened)
at::Tensor silu_mul(const at::Tensor& g, const at::Tensor& u) {
  TB_CHECK_CUDA(g);
  TORCH_CHECK(g.sizes() == u.sizes() && g.scalar_type() == u.scalar_type(), "silu_mul: same shape and dtype");
  const at::cuda::CUDAGuard guard(g.device());
  at::Tensor gc = contig16(g), uc = contig16(u);
  at::Tensor h = at::empty_like(gc);
  const int64_t F = gc.dim() ? gc.size(-1) : 1;
  const int64_t M = F ? gc.numel() / F : 0;
  TB_DISPATCH_FLOAT(gc.scalar_type(), "silu_mul", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(F % V == 0, "silu_mul: the last dim must be a multiple of ", V);
    const int64_t n = M * (F / V);
    if (n) swiglu_fwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
               (const scalar_t*)gc.data_ptr(), F, (const scalar_t*)uc.data_ptr(), F, (scalar_t*)h.data_ptr(), M,
               (int)F);
  });
  check_launch("silu_mul");
  return h;
}

at::Tensor swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu) {
  TB_CHECK_CUDA(gu);
  const at::cuda::CUDAGuard g(gu.device());
  at::Tensor x = contig16(gu), d = contig16(dh);
  const int64_t M = x.size(0);
  const int F = x.size(1) / 2;
  at::Tensor dgu = at::empty_like(x);
  TB_DISPATCH_FLOAT(x.scalar_type(), "swiglu_bwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    const int64_t n = M * (F / V);
    if (n) swiglu_bwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
        (const scalar_t*)d.data_ptr(), (const scalar_t*)x.data_ptr(), (scalar_t*)dgu.data_ptr(), M, F);
  });
  check_launch("swiglu_bwd");
  return dgu;
}

// ------------------------------------------------------ memory epilogues
// a = act(z)   (z kept for the backward)
template <typename T>
__global__ void act_kernel(const T* __restrict__ z, T* __restrict__ a, int64_t nvec, int act) {
  constexpr int V = Vec16<T>::N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float v[V];
    load16<T>(z + i * V, v);
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = act_f(act, v[k]);
    store16<T>(a + i * V, v);
  }
}

// g <- g * act'(z)  (in place)
template <typename T>
__global__ void act_grad_mul_kernel(T* __restrict__ g, const T* __restrict__ z, int64_t nvec, int act) {
  constexpr int V = Vec16<T>::N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float gv[V], zv[V];
    load16<T>(g + i * V, gv);
    load16<T>(z + i * V, zv);
#pragma unroll
    for (int k = 0; k < V; ++k) gv[k] *= act_grad_f(act, zv[k]);
    store16<T>(g + i * V, gv);
  }
}

// out <- g * act'(z)  (out of place: the autograd backward of an activation)
template <typename T>
__global__ void act_grad_out_kernel(const T* __restrict__ g, const T* __restrict__ z, T* __restrict__ out,
                                    int64_t nvec, int act) {
  constexpr int V = Vec16<T>::N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float gv[V], zv[V];
    load16<T>(g + i * V, gv);
    load16<T>(z + i * V, zv);
#pragma unroll
    for (int k = 0; k < V; ++k) gv[k] *= act_grad_f(act, zv[k]);
    store16<T>(out + i * V, gv);
  }
}

// d <- (p - v) * scale   (in place on p)
template <typename T>
__global__ void scaled_err_kernel(T* __restrict__ p, const T* __restrict__ v, int64_t nvec, float scale) {
  constexpr int V = Vec16<T>::N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    float a[V], b[V];
    load16<T>(p + i * V, a);
    load16<T>(v + i * V, b);
#pragma unroll
    for (int k = 0; k < V; ++k) a[k] = (a[k] - b[k]) * scale;
    store16<T>(p + i * V, a);
  }
}

// gates[0..2] = alpha, theta, eta.  m' = eta*m - theta*G ; w' = (1-alpha)*w + m'
template <typename T, typename G>
__global__ void mem_update_kernel(const T* __restrict__ w, const T* __restrict__ m, const G* __restrict__ grad,
                                  T* __restrict__ w_out, T* __restrict__ m_out, const float* __restrict__ gates,
                                  int64_t n) {
  const float alpha = gates[0], theta = gates[1], eta = gates[2];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    // round the momentum to the state dtype before it enters the weight
    // update, as the reference does when it builds S then W in that dtype
    const float s = to_f<T>(from_f<T>(eta * to_f<T>(m[i]) - theta * to_f<G>(grad[i])));
    m_out[i] = from_f<T>(s);
    w_out[i] = from_f<T>((1.f - alpha) * to_f<T>(w[i]) + s);
  }
}

// ------------------------------------------------------------ gates
// partial sums of x over T: part[s, b, d] for split s of the sequence
template <typename T>
__global__ void seq_sum_kernel(const T* __restrict__ x, int64_t sb, int64_t st, float* __restrict__ part, int B,
                               int Tn, int D, int splits) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y, s = blockIdx.z;
  if (d >= D) return;
  const int per = (Tn + splits - 1) / splits;
  const int t0 = s * per, t1 = min(Tn, t0 + per);
  float acc = 0.f;
  const T* p = x + (int64_t)b * sb + d;
  for (int t = t0; t < t1; ++t) acc += to_f<T>(p[(int64_t)t * st]);
  part[((int64_t)s * B + b) * D + d] = acc;
}

// xm[b, d] = mean over the sequence (sum of the split partials), rounded to the
// input dtype as x.mean() in that dtype does.  Done once, not per GEMV block.
template <typename T>
__global__ void seq_mean_finish_kernel(const float* __restrict__ part, int splits, float* __restrict__ xm, int BD,
                                       int Tn) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= BD) return;
  float s = 0.f;
  for (int k = 0; k < splits; ++k) s += part[(int64_t)k * BD + e];
  xm[e] = to_f<T>(from_f<T>(s / (float)Tn));
}

// grid (ceil(D / 32), 3 gates), 8 warps of 4 output features each; the lanes
// stream W[o, :] in 16-byte pieces against the B sequence means (read through
// L1 as float4), eight samples at a time.
// sig_part[gate, blk] = sum over (b, o in blk) sigmoid(z)
template <typename T>
__global__ void gate_gemv_kernel(const float* __restrict__ xm, const T* __restrict__ W0, const T* __restrict__ W1,
                                 const T* __restrict__ W2, const T* __restrict__ b0, const T* __restrict__ b1,
                                 const T* __restrict__ b2, float* __restrict__ sig_part, int B, int D) {
  constexpr int V = Vec16<T>::N;
  constexpr int ROWS = 4;
  const int gate = blockIdx.y;
  const T* W = gate == 0 ? W0 : (gate == 1 ? W1 : W2);
  const T* bb = gate == 0 ? b0 : (gate == 1 ? b1 : b2);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float local = 0.f;
  for (int r = 0; r < ROWS; ++r) {
    const int o = (blockIdx.x * nw + wid) * ROWS + r;
    if (o >= D) break;
    const T* wr = W + (int64_t)o * D;
    const float bias = bb ? to_f<T>(bb[o]) : 0.f;
    for (int bs = 0; bs < B; bs += 8) {
      const int nb = min(8, B - bs);
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int d = lane * V; d < D; d += 32 * V) {
        float w[V];
        load16<T>(wr + d, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < nb) {
            const float4* xr = reinterpret_cast<const float4*>(xm + (int64_t)(bs + j) * D + d);
#pragma unroll
            for (int v4 = 0; v4 < V / 4; ++v4) {
              const float4 q = __ldg(xr + v4);
              acc[j] += w[4 * v4] * q.x + w[4 * v4 + 1] * q.y + w[4 * v4 + 2] * q.z + w[4 * v4 + 3] * q.w;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j < nb) {
          const float z = warp_sum(acc[j]) + bias;
          // round the logit to the input dtype, as the reference's Linear output is
          if (lane == 0) local += sigmoidf_(to_f<T>(from_f<T>(z)));
        }
      }
    }
  }
  __shared__ float red[32];
  if (lane == 0) red[wid] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < nw; ++k) s += red[k];
    sig_part[gate * gridDim.x + blockIdx.x] = s;
  }
}

__global__ void gate_finish_kernel(const float* __restrict__ sig_part, int nblk, int B, int D, float lr, float mom,
                                   float* __restrict__ gates) {
  const int g = threadIdx.x;
  if (g >= 3) return;
  float s = 0.f;
  for (int k = 0; k < nblk; ++k) s += sig_part[g * nblk + k];
  float mean = s / (float)(B * D);
  gates[g] = g == 0 ? mean : (g == 1 ? mean * lr : mean * mom);
}

// Host: gates of the reference memory for x [B, T, D]; returns float[3] on device.
at::Tensor memory_gates(const at::Tensor& x, const std::vector<at::Tensor>& ws, const std::vector<at::Tensor>& bs,
                        double lr, double mom) {
  TB_CHECK_CUDA(x);
  const at::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 3 && ws.size() == 3 && bs.size() == 3, "memory_gates: bad arguments");
  const int B = x.size(0), Tn = x.size(1), D = x.size(2);
  const int splits = std::max(1, std::min(64, Tn / 64));
  at::Tensor part = at::empty({splits, B, D}, x.options().dtype(at::kFloat));
  at::Tensor gates = at::empty({3}, x.options().dtype(at::kFloat));
  const int nblk = (D + 31) / 32;  // 8 warps per block, 4 output features per warp
  at::Tensor sig = at::empty({3, nblk}, x.options().dtype(at::kFloat));
  TB_DISPATCH_FLOAT(x.scalar_type(), "memory_gates", [&] {
    using T = scalar_t;
    std::vector<at::Tensor> wc(3), bc(3);
    for (int i = 0; i < 3; ++i) {
      wc[i] = ws[i].to(x.scalar_type()).contiguous();
      bc[i] = bs[i].defined() ? bs[i].to(x.scalar_type()).contiguous() : at::Tensor();
    }
    dim3 g1((D + 127) / 128, B, splits);
    seq_sum_kernel<T><<<g1, 128, 0, stream()>>>((const T*)x.data_ptr(), x.stride(0), x.stride(1),
                                                 part.data_ptr<float>(), B, Tn, D, splits);
    TORCH_CHECK(D % Vec16<T>::N == 0, "memory_gates: dim must be a multiple of ", Vec16<T>::N);
    at::Tensor xm = at::empty({B, D}, x.options().dtype(at::kFloat));
    seq_mean_finish_kernel<T><<<(B * D + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), splits,
                                                                        xm.data_ptr<float>(), B * D, Tn);
    dim3 g2(nblk, 3);
    gate_gemv_kernel<T><<<g2, 256, 0, stream()>>>(
        xm.data_ptr<float>(), (const T*)wc[0].data_ptr(), (const T*)wc[1].data_ptr(),
        (const T*)wc[2].data_ptr(), bc[0].defined() ? (const T*)bc[0].data_ptr() : nullptr,
        bc[1].defined() ? (const T*)bc[1].data_ptr() : nullptr, bc[2].defined() ? (const T*)bc[2].data_ptr() : nullptr,
        sig.data_ptr<float>(), B, D);
    gate_finish_kernel<<<1, 32, 0, stream()>>>(sig.data_ptr<float>(), nblk, B, D, (float)lr, (float)mom,
                                               gates.data_ptr<float>());
  });
  check_launch("memory_gates");
  return gates;
}

void act_inplace(const at::Tensor& z, at::Tensor& a, const std::string& act) {
  const at::cuda::CUDAGuard g(z.device());
  TORCH_CHECK(z.is_contiguous() && a.is_contiguous() && aligned16(z) && aligned16(a), "act: contiguous aligned tensors required");
  TB_DISPATCH_FLOAT(z.scalar_type(), "act", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(z.numel() % V == 0, "act: numel must be a multiple of ", V);
    const int64_t n = z.numel() / V;
    if (n) act_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>((const scalar_t*)z.data_ptr(), (scalar_t*)a.data_ptr(), n, act_code(act));
  });
  check_launch("act");
}

void act_grad_mul(at::Tensor& gr, const at::Tensor& z, const std::string& act) {
  const at::cuda::CUDAGuard g(z.device());
  TORCH_CHECK(z.is_contiguous() && gr.is_contiguous() && aligned16(z) && aligned16(gr), "act_grad_mul: contiguous aligned tensors required");
  TB_DISPATCH_FLOAT(z.scalar_type(), "act_grad_mul", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    const int64_t n = z.numel() / V;
    if (n) act_grad_mul_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>((scalar_t*)gr.data_ptr(), (const scalar_t*)z.data_ptr(), n, act_code(act));
  });
  check_launch("act_grad_mul");
}

void act_grad_out(const at::Tensor& g, const at::Tensor& z, at::Tensor& out, const std::string& act) {
  const at::cuda::CUDAGuard guard(z.device());
  TORCH_CHECK(z.is_contiguous() && g.is_contiguous() && out.is_contiguous() && aligned16(z) && aligned16(g) &&
                  aligned16(out) && g.numel() == z.numel() && out.numel() == z.numel() &&
                  g.scalar_type() == z.scalar_type() && out.scalar_type() == z.scalar_type(),
              "act_grad_out: contiguous aligned tensors of one shape and dtype required");
  TB_DISPATCH_FLOAT(z.scalar_type(), "act_grad_out", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(z.numel() % V == 0, "act_grad_out: numel must be a multiple of ", V);
    const int64_t n = z.numel() / V;
    if (n)
      act_grad_out_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
          (const scalar_t*)g.data_ptr(), (const scalar_t*)z.data_ptr(), (scalar_t*)out.data_ptr(), n, act_code(act));
  });
  check_launch("act_grad_out");
}

void scaled_err(at::Tensor& p, const at::Tensor& v, double scale) {
  const at::cuda::CUDAGuard g(p.device());
  TORCH_CHECK(p.is_contiguous() && v.is_contiguous() && aligned16(p) && aligned16(v), "scaled_err: contiguous aligned tensors required");
  TB_DISPATCH_FLOAT(p.scalar_type(), "scaled_err", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    TORCH_CHECK(p.numel() % V == 0, "scaled_err: numel must be a multiple of ", V);
    const int64_t n = p.numel() / V;
    if (n) scaled_err_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>((scalar_t*)p.data_ptr(), (const scalar_t*)v.data_ptr(), n, (float)scale);
  });
  check_launch("scaled_err");
}

std::vector<at::Tensor> mem_update(const at::Tensor& w, const at::Tensor& m, const at::Tensor& grad,
                                   const at::Tensor& gates) {
  const at::cuda::CUDAGuard g(w.device());
  at::Tensor wc = w.contiguous(), mc = m.contiguous(), gc = grad.contiguous();
  at::Tensor w_out = at::empty_like(wc), m_out = at::empty_like(mc);
  const int64_t n = wc.numel();
  TB_DISPATCH_FLOAT(wc.scalar_type(), "mem_update", [&] {
    using T = scalar_t;
    if (gc.scalar_type() == at::kFloat) {
      mem_update_kernel<T, float><<<ew_blocks(n), 256, 0, stream()>>>(
          (const T*)wc.data_ptr(), (const T*)mc.data_ptr(), gc.data_ptr<float>(), (T*)w_out.data_ptr(),
          (T*)m_out.data_ptr(), gates.data_ptr<float>(), n);
    } else {
      TORCH_CHECK(gc.scalar_type() == wc.scalar_type(), "mem_update: grad dtype");
      mem_update_kernel<T, T><<<ew_blocks(n), 256, 0, stream()>>>(
          (const T*)wc.data_ptr(), (const T*)mc.data_ptr(), (const T*)gc.data_ptr(), (T*)w_out.data_ptr(),
          (T*)m_out.data_ptr(), gates.data_ptr<float>(), n);
    }
  });
  check_launch("mem_update");
  return {w_out, m_out};
}

}  // namespace tb
