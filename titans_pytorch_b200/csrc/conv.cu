// Causal depthwise conv1d + bias + SiLU (+ row L2-normalisation), forward and
// backward, written for memory-level parallelism.
//
// Forward / backward-A: a thread owns one (row, 16-byte column slice); the K
// input rows it needs are independent loads (clamped address, zeroed when
// before t = 0), so all of them are in flight at once and neighbouring rows'
// re-reads hit L1/L2.  A block is RB rows x TPR threads (TPR = the threads of
// one row, a multiple of 32), so the per-row L2-norm reduction is a warp
// shuffle plus a few shared-memory adds.
//
// Backward-B: dx by the transposed convolution of dc, and the dw/db column
// sums; each thread walks a time range U rows at a time with all 2*(U+K-1)
// loads of a step issued before any use, keeping the partial sums in
// registers; block partials are reduced in a fixed order (deterministic).
#include "common.cuh"

namespace tb {

constexpr float kL2Eps = 1e-12f;  // F.normalize default eps

// N consecutive fp32 values starting at column col (N a multiple of 4, col
// 4-aligned) with float4 loads; zeros when p is null.
template <int N>
__device__ __forceinline__ void load_cols_f32(const float* __restrict__ p, int col, float (&o)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    if (p) {
      const float4 v = *reinterpret_cast<const float4*>(p + col + i);
      o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
    } else {
      o[i] = o[i + 1] = o[i + 2] = o[i + 3] = 0.f;
    }
  }
}

// Weights in the parameter's own layout and dtype: w[d][j] ([D, K], the
// Conv1d weight [D, 1, K] viewed), so no transposed fp32 copy is made per
// call.  The KS taps of V consecutive columns are KS*V contiguous elements,
// read as 16-byte pieces (the column start is a multiple of V).
template <typename T, int KS>
__device__ __forceinline__ void load_taps(const T* __restrict__ w, int col, float (&o)[KS][Vec16<T>::N]) {
  constexpr int V = Vec16<T>::N;
  constexpr int NB = KS * V * (int)sizeof(T);
  const T* src = w + (int64_t)col * KS;
  if constexpr (NB % 16 == 0) {
    uint4 buf[NB / 16];
#pragma unroll
    for (int i = 0; i < NB / 16; ++i) buf[i] = reinterpret_cast<const uint4*>(src)[i];
    const T* e = reinterpret_cast<const T*>(buf);
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int j = 0; j < KS; ++j) o[j][i] = to_f<T>(e[i * KS + j]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int j = 0; j < KS; ++j) o[j][i] = to_f<T>(src[i * KS + j]);
  }
}

template <typename T>
__device__ __forceinline__ void load_bias(const T* __restrict__ b, int col, float (&o)[Vec16<T>::N]) {
  constexpr int V = Vec16<T>::N;
  if (b) {
    load16<T>(b + col, o);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = 0.f;
  }
}

template <typename T, int KS>
__global__ void __launch_bounds__(512) conv_fwd_rows(const T* __restrict__ x, int64_t sb, int64_t st,
                                                     const T* __restrict__ wt, const T* __restrict__ bias,
                                                     T* __restrict__ y, int64_t rows, int Tn, int D, bool normalize) {
  constexpr int V = Vec16<T>::N;
  __shared__ float red[32][33];
  const int tpr = blockDim.x, lane = threadIdx.x & 31, wir = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
  const int col = threadIdx.x * V;
  const bool active = col < D && r < rows;
  float o[V];
  float ss = 0.f;
  if (active) {
    const int b = (int)(r / Tn), t = (int)(r % Tn);
    const T* xb = x + (int64_t)b * sb + col;
    float xv[KS][V];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const int tt = t - KS + 1 + j;
      load16<T>(xb + (int64_t)max(tt, 0) * st, xv[j]);
      if (tt < 0)
#pragma unroll
        for (int i = 0; i < V; ++i) xv[j][i] = 0.f;
    }
    float acc[V];
    load_bias<T>(bias, col, acc);
    if (wt) {
      float wj[KS][V];
      load_taps<T, KS>(wt, col, wj);
#pragma unroll
      for (int j = 0; j < KS; ++j)
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += wj[j][i] * xv[j][i];
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += xv[KS - 1][i];
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      o[i] = silu_(acc[i]);
      ss += o[i] * o[i];
    }
  }
  float inv = 1.f;
  if (normalize) {
    ss = warp_sum(ss);
    if (lane == 0) red[threadIdx.y][wir] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int k = 0; k < (tpr >> 5); ++k) tot += red[threadIdx.y][k];
    inv = 1.f / fmaxf(sqrtf(tot), kL2Eps);
  }
  if (active) {
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] *= inv;
    store16<T>(y + r * D + col, o);
  }
}

// R consecutive tokens of one sequence per thread (Tn % R == 0): the R + KS - 1
// input rows are loaded once (instead of KS times each), the taps and the bias
// once per thread, and the R row norms share one block reduction.
template <typename T, int KS, int R>
__global__ void __launch_bounds__(256) conv_fwd_rrows(const T* __restrict__ x, int64_t sb, int64_t st,
                                                      const T* __restrict__ wt, const T* __restrict__ bias,
                                                      T* __restrict__ y, int64_t rows, int Tn, int D, bool normalize) {
  constexpr int V = Vec16<T>::N;
  __shared__ float red[8][R][8];  // [row group][row][warp of the row]
  const int nw = blockDim.x >> 5, lane = threadIdx.x & 31, wir = threadIdx.x >> 5;
  const int64_t r0 = ((int64_t)blockIdx.x * blockDim.y + threadIdx.y) * R;
  const int col = threadIdx.x * V;
  const bool active = col < D && r0 < rows;
  float o[R][V];
  float ss[R];
#pragma unroll
  for (int k = 0; k < R; ++k) ss[k] = 0.f;
  if (active) {
    const int b = (int)(r0 / Tn), t0 = (int)(r0 % Tn);
    const T* xb = x + (int64_t)b * sb + col;
    float xin[R + KS - 1][V];  // xin[i] = x[t0 - KS + 1 + i]
#pragma unroll
    for (int i = 0; i < R + KS - 1; ++i) {
      const int tt = t0 - KS + 1 + i;
      load16<T>(xb + (int64_t)max(tt, 0) * st, xin[i]);
      if (tt < 0)
#pragma unroll
        for (int e = 0; e < V; ++e) xin[i][e] = 0.f;
    }
    float bv[V];
    load_bias<T>(bias, col, bv);
    float wj[KS][V];
    if (wt) load_taps<T, KS>(wt, col, wj);
#pragma unroll
    for (int k = 0; k < R; ++k) {
#pragma unroll
      for (int e = 0; e < V; ++e) {
        float acc = bv[e];
        if (wt) {
#pragma unroll
          for (int j = 0; j < KS; ++j) acc += wj[j][e] * xin[k + j][e];
        } else {
          acc += xin[k + KS - 1][e];
        }
        o[k][e] = silu_(acc);
        ss[k] += o[k][e] * o[k][e];
      }
    }
  }
  float inv[R];
#pragma unroll
  for (int k = 0; k < R; ++k) inv[k] = 1.f;
  if (normalize) {
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const float v = warp_sum(ss[k]);
      if (lane == 0) red[threadIdx.y][k][wir] = v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < R; ++k) {
      float tot = 0.f;
      for (int w = 0; w < nw; ++w) tot += red[threadIdx.y][k][w];
      inv[k] = 1.f / fmaxf(sqrtf(tot), kL2Eps);
    }
  }
  if (active) {
#pragma unroll
    for (int k = 0; k < R; ++k) {
#pragma unroll
      for (int e = 0; e < V; ++e) o[k][e] *= inv[k];
      store16<T>(y + (r0 + k) * D + col, o[k]);
    }
  }
}

// dc = d(loss)/d(conv output) (fp32, [rows, D]); without a conv it writes dx directly.
template <typename T, int KS>
__global__ void __launch_bounds__(512) conv_bwd_a_rows(const T* __restrict__ dy, const T* __restrict__ x,
                                                       int64_t sb, int64_t st, const T* __restrict__ wt,
                                                       const T* __restrict__ bias, float* __restrict__ dc,
                                                       T* __restrict__ dx_direct, int64_t rows, int Tn, int D,
                                                       bool normalize) {
  constexpr int V = Vec16<T>::N;
  __shared__ float red_s[32][33], red_d[32][33];
  const int tpr = blockDim.x, lane = threadIdx.x & 31, wir = threadIdx.x >> 5;
  const int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
  const int col = threadIdx.x * V;
  const bool active = col < D && r < rows;
  float pre[V], g[V];
  float ss = 0.f, sd = 0.f;
  if (active) {
    const int b = (int)(r / Tn), t = (int)(r % Tn);
    const T* xb = x + (int64_t)b * sb + col;
    float xv[KS][V];
#pragma unroll
    for (int j = 0; j < KS; ++j) {
      const int tt = t - KS + 1 + j;
      load16<T>(xb + (int64_t)max(tt, 0) * st, xv[j]);
      if (tt < 0)
#pragma unroll
        for (int i = 0; i < V; ++i) xv[j][i] = 0.f;
    }
    load16<T>(dy + r * D + col, g);
    load_bias<T>(bias, col, pre);
    if (wt) {
      float wj[KS][V];
      load_taps<T, KS>(wt, col, wj);
#pragma unroll
      for (int j = 0; j < KS; ++j)
#pragma unroll
        for (int i = 0; i < V; ++i) pre[i] += wj[j][i] * xv[j][i];
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) pre[i] += xv[KS - 1][i];
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float s = silu_(pre[i]);
      ss += s * s;
      sd += s * g[i];
    }
  }
  float den = 1.f, coef = 0.f;
  if (normalize) {
    ss = warp_sum(ss);
    sd = warp_sum(sd);
    if (lane == 0) { red_s[threadIdx.y][wir] = ss; red_d[threadIdx.y][wir] = sd; }
    __syncthreads();
    float ts = 0.f, td = 0.f;
    for (int k = 0; k < (tpr >> 5); ++k) { ts += red_s[threadIdx.y][k]; td += red_d[threadIdx.y][k]; }
    const float nrm = sqrtf(ts);
    den = fmaxf(nrm, kL2Eps);
    coef = nrm > kL2Eps ? td / (den * den) : 0.f;
  }
  if (active) {
    float o[V];
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = (g[i] - silu_(pre[i]) * coef) / den * silu_grad_(pre[i]);
    if (dc != nullptr) {
#pragma unroll
      for (int i = 0; i < V; i += 4)
        *reinterpret_cast<float4*>(dc + r * D + col + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    } else {
      store16<T>(dx_direct + r * D + col, o);
    }
  }
}

// grid (splits, B, column groups): dx[t] = sum_j w[j] dc[t+KS-1-j];
// dw[j] += dc[t] x[t-KS+1+j]; db += dc[t].  part: [splits*B][KS+1][D]
template <typename T, int KS, int U>
__global__ void __launch_bounds__(256) conv_bwd_b_rows(const float* __restrict__ dc, const T* __restrict__ x,
                                                       int64_t sb, int64_t st, const T* __restrict__ wt,
                                                       T* __restrict__ dx, float* __restrict__ part, int Tn, int D,
                                                       int rows_per_split) {
  constexpr int V = Vec16<T>::N;
  constexpr int NR = U + KS - 1;
  const int b = blockIdx.y, sp = blockIdx.x;
  const int col = (blockIdx.z * blockDim.x + threadIdx.x) * V;
  if (col >= D) return;
  const int ts = sp * rows_per_split, te = min(Tn, ts + rows_per_split);
  const T* xb = x + (int64_t)b * sb + col;
  const float* dcb = dc + (int64_t)b * Tn * D + col;
  float w[KS][V], aw[KS][V], ab[V];
  load_taps<T, KS>(wt, col, w);
#pragma unroll
  for (int j = 0; j < KS; ++j)
#pragma unroll
    for (int i = 0; i < V; ++i) aw[j][i] = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) ab[i] = 0.f;
  for (int t0 = ts; t0 < te; t0 += U) {
    // rows needed: dc[t0 .. t0+U+KS-2] (zero past the end), x[t0-KS+1 .. t0+U-1] (zero before 0)
    float dv[NR][V], xv[NR][V];
#pragma unroll
    for (int k = 0; k < NR; ++k) {
      const int td = t0 + k;
      const float* p = dcb + (int64_t)min(td, Tn - 1) * D;
      const bool z = td >= Tn;
#pragma unroll
      for (int i = 0; i < V; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(p + i);
        dv[k][i] = z ? 0.f : v.x;
        dv[k][i + 1] = z ? 0.f : v.y;
        dv[k][i + 2] = z ? 0.f : v.z;
        dv[k][i + 3] = z ? 0.f : v.w;
      }
      const int tx = t0 - KS + 1 + k;
      load16<T>(xb + (int64_t)min(max(tx, 0), Tn - 1) * st, xv[k]);
      if (tx < 0 || tx >= Tn)
#pragma unroll
        for (int i = 0; i < V; ++i) xv[k][i] = 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = t0 + u;
      if (t >= te) break;
      float o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          a += w[j][i] * dv[u + KS - 1 - j][i];  // dc[t + KS - 1 - j]
          aw[j][i] += dv[u][i] * xv[u + j][i];    // dc[t] * x[t - KS + 1 + j]
        }
        o[i] = a;
        ab[i] += dv[u][i];
      }
      store16<T>(dx + ((int64_t)b * Tn + t) * D + col, o);
    }
  }
  if (part == nullptr) return;
  float* pp = part + ((int64_t)(sp * gridDim.y + b)) * (KS + 1) * D + col;
#pragma unroll
  for (int j = 0; j < KS; ++j)
#pragma unroll
    for (int i = 0; i < V; ++i) pp[(int64_t)j * D + i] = aw[j][i];
#pragma unroll
  for (int i = 0; i < V; ++i) pp[(int64_t)KS * D + i] = ab[i];
}

// out[i] = sum_g part[g, i]: block (32 columns x 8 row groups); each thread
// sums every 8th row of its column, then the 8 partials are added in a fixed
// order (deterministic).
__global__ void colsum_kernel2(const float* __restrict__ part, float* __restrict__ out, int G, int64_t N) {
  __shared__ float red[8][33];
  const int64_t i = (int64_t)blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (i < N)
    for (int g = threadIdx.y; g < G; g += 8) s += part[(int64_t)g * N + i];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && i < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][threadIdx.x];
    out[i] = t;
  }
}

#define TB_KS_SWITCH(KV, ...)                                  \
  switch (KV) {                                                \
    case 1: { constexpr int KS = 1; __VA_ARGS__; break; }      \
    case 2: { constexpr int KS = 2; __VA_ARGS__; break; }      \
    case 3: { constexpr int KS = 3; __VA_ARGS__; break; }      \
    case 4: { constexpr int KS = 4; __VA_ARGS__; break; }      \
    case 5: { constexpr int KS = 5; __VA_ARGS__; break; }      \
    case 6: { constexpr int KS = 6; __VA_ARGS__; break; }      \
    case 7: { constexpr int KS = 7; __VA_ARGS__; break; }      \
    case 8: { constexpr int KS = 8; __VA_ARGS__; break; }      \
    default: TORCH_CHECK(false, "conv kernel size must be 1..8"); \
  }

#define TB_DISPATCH_BF16_F32(dtype, NAME, ...)                  \
  [&] {                                                         \
    if ((dtype) == at::kBFloat16) {                             \
      using scalar_t = __nv_bfloat16;                           \
      return __VA_ARGS__();                                     \
    } else if ((dtype) == at::kFloat) {                         \
      using scalar_t = float;                                   \
      return __VA_ARGS__();                                     \
    }                                                           \
    TORCH_CHECK(false, NAME, ": bf16 or fp32 only, got ", dtype); \
  }()

// [D, 1, K] Conv1d weight -> [D, K] in the activation dtype (a view when it
// already is contiguous and of that dtype, as model parameters are)
static at::Tensor conv_wt(const c10::optional<at::Tensor>& w, int D, at::ScalarType dt) {
  if (!w.has_value() || !w->defined()) return at::Tensor();
  at::Tensor t = w->reshape({D, -1}).to(dt).contiguous();
  TORCH_CHECK(aligned16(t), "conv_silu_norm: weight must be 16-byte aligned");
  return t;
}
static at::Tensor conv_bias(const c10::optional<at::Tensor>& b, at::ScalarType dt) {
  if (!b.has_value() || !b->defined()) return at::Tensor();
  at::Tensor t = b->to(dt).contiguous();
  TORCH_CHECK(aligned16(t), "conv_silu_norm: bias must be 16-byte aligned");
  return t;
}

static void check_x(const at::Tensor& x, int V) {
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "conv_silu_norm: x must be [B, T, D] with a contiguous last dim");
  const int D = x.size(2);
  TORCH_CHECK(D % V == 0 && x.stride(1) % V == 0 && x.stride(0) % V == 0 && aligned16(x),
              "conv_silu_norm: D, row strides and base must be 16-byte multiples");
  TORCH_CHECK(D / V <= 512, "conv_silu_norm: D too large (at most 512 16-byte slices per row)");
}

static int threads_for(int D, int V) { return ((D / V) + 31) / 32 * 32; }
static dim3 row_block(int tpr) { return dim3(tpr, std::max(1, std::min(32, 256 / tpr))); }

at::Tensor conv_silu_norm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w,
                              const c10::optional<at::Tensor>& b, bool normalize) {
  TB_CHECK_CUDA(x);
  const at::cuda::CUDAGuard g(x.device());
  const int B = x.size(0), Tn = x.size(1), D = x.size(2);
  at::Tensor wt = conv_wt(w, D, x.scalar_type());
  const int K = wt.defined() ? wt.size(1) : 1;
  at::Tensor bias = conv_bias(b, x.scalar_type());
  at::Tensor y = at::empty({B, Tn, D}, x.options());
  const int64_t rows = (int64_t)B * Tn;
  if (rows == 0) return y;
  TB_DISPATCH_BF16_F32(x.scalar_type(), "conv_silu_norm_fwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    check_x(x, V);
    const int tpr = threads_for(D, V);
    constexpr int R = 4;
    if (Tn % R == 0 && tpr <= 256) {
      const dim3 blk(tpr, std::max(1, std::min(8, 256 / tpr)));
      const int64_t grid = (rows / R + blk.y - 1) / blk.y;
      TB_KS_SWITCH(K, conv_fwd_rrows<scalar_t, KS, R><<<grid, blk, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1),
          wt.defined() ? (const scalar_t*)wt.data_ptr() : nullptr,
          bias.defined() ? (const scalar_t*)bias.data_ptr() : nullptr, (scalar_t*)y.data_ptr(), rows, Tn, D,
          normalize));
    } else {
      const dim3 blk = row_block(tpr);
      const int64_t grid = (rows + blk.y - 1) / blk.y;
      TB_KS_SWITCH(K, conv_fwd_rows<scalar_t, KS><<<grid, blk, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1),
          wt.defined() ? (const scalar_t*)wt.data_ptr() : nullptr,
          bias.defined() ? (const scalar_t*)bias.data_ptr() : nullptr, (scalar_t*)y.data_ptr(), rows, Tn, D,
          normalize));
    }
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
  at::Tensor dyc = contig16(dy.to(x.scalar_type()));
  at::Tensor wt = conv_wt(w, D, x.scalar_type());
  const int K = wt.defined() ? wt.size(1) : 1;
  at::Tensor bias = conv_bias(b, x.scalar_type());
  at::Tensor dx = at::empty({B, Tn, D}, x.options());
  at::Tensor dw = at::empty({0}, x.options().dtype(at::kFloat)), db = at::empty({0}, x.options().dtype(at::kFloat));
  const int64_t rows = (int64_t)B * Tn;
  if (rows == 0) return {dx.zero_(), dw, db};
  at::Tensor dc = wt.defined() ? at::empty({B, Tn, D}, x.options().dtype(at::kFloat)) : at::Tensor();
  TB_DISPATCH_BF16_F32(x.scalar_type(), "conv_silu_norm_bwd", [&] {
    constexpr int V = Vec16<scalar_t>::N;
    check_x(x, V);
    const int tpr = threads_for(D, V);
    const dim3 blk = row_block(tpr);
    const int64_t grid = (rows + blk.y - 1) / blk.y;
    TB_KS_SWITCH(K, conv_bwd_a_rows<scalar_t, KS><<<grid, blk, 0, stream()>>>(
        (const scalar_t*)dyc.data_ptr(), (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1),
        wt.defined() ? (const scalar_t*)wt.data_ptr() : nullptr, bias.defined() ? (const scalar_t*)bias.data_ptr() : nullptr,
        dc.defined() ? dc.data_ptr<float>() : nullptr, (scalar_t*)dx.data_ptr(), rows, Tn, D, normalize));
    check_launch("conv_silu_norm_bwd_a");
    if (wt.defined()) {
      const int want_warps = num_sms() * 12;
      int splits = std::max(1, want_warps / std::max(1, B * (tpr / 32)));
      splits = std::min(splits, std::max(1, Tn / 8));
      const int rps = (Tn + splits - 1) / splits;
      splits = (Tn + rps - 1) / rps;
      at::Tensor part = need_wgrad ? at::empty({splits * B, K + 1, D}, x.options().dtype(at::kFloat)) : at::Tensor();
      const int bx = std::min(tpr, 256);
      dim3 g2(splits, B, (tpr + bx - 1) / bx);
      TB_KS_SWITCH(K, conv_bwd_b_rows<scalar_t, KS, 2><<<g2, bx, 0, stream()>>>(
          dc.data_ptr<float>(), (const scalar_t*)x.data_ptr(), x.stride(0), x.stride(1), (const scalar_t*)wt.data_ptr(),
          (scalar_t*)dx.data_ptr(), need_wgrad ? part.data_ptr<float>() : nullptr, Tn, D, rps));
      check_launch("conv_silu_norm_bwd_b");
      if (need_wgrad) {
        at::Tensor red = at::empty({K + 1, D}, x.options().dtype(at::kFloat));
        const int64_t N = (int64_t)(K + 1) * D;
        colsum_kernel2<<<(N + 31) / 32, dim3(32, 8), 0, stream()>>>(part.data_ptr<float>(), red.data_ptr<float>(),
                                                                    splits * B, N);
        check_launch("conv_silu_norm_bwd colsum");
        dw = red.narrow(0, 0, K).t().contiguous();  // [D, K]
        db = red[K].contiguous();
      }
    }
  });
  return {dx, dw, db};
}

}  // namespace tb
