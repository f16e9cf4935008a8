// Windowed causal attention with always-visible prefix keys.
//
//   pack:    fused qkv [B, T, 3D] (+ prefix kv [Bp, P, 2D]) -> Q [B,H,T,d],
//            K/V [B,H,P+T,d] with interleaved-pair RoPE applied (query i at
//            position P+i, key j at position j), prefix rows first.
//   forward: flash-style online softmax; a query block visits only the key
//            tiles that hold prefix keys or main keys inside its window, so
//            the work is O(T * (P + window)) and no mask tensor exists.
//            Writes O [B, T, H, d] (ready for the output projection) and the
//            per-row log-sum-exp.
//   backward: one CTA per (key tile, query range); dK/dV accumulate in
//            registers, dQ through fp32 vector reductions (red.global.add),
//            long query ranges (the prefix tile sees every query) are split
//            across CTAs.  unpack applies the inverse rotation and writes the
//            gradient back into the fused-qkv layout (+ prefix kv).
//
// Tensor-core path: mma.sync m16n8k16 bf16 with fp32 accumulation, operands
// staged in XOR-swizzled shared memory by cp.async and read with ldmatrix.
#include "common.cuh"

namespace tb {
namespace attn {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(p), "f"(a), "f"(b) : "memory");
}

// Shared-memory tile of ROWS x (RS*8) bf16, 16-byte chunks XOR-swizzled by row
// within groups of 8 chunks so ldmatrix row reads hit distinct banks.
template <int RS>
__device__ __forceinline__ int swz(int row, int col) {
  const int ch = col >> 3;
  return row * RS * 8 + (((ch & ~7) | ((ch ^ row) & 7)) << 3) + (col & 7);
}

// Copy `rows` rows of HD bf16 from global (row stride gstride elements) into a
// swizzled tile; rows >= nvalid are zero-filled.
template <int HD, int RS, int ROWS, int NT>
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, int64_t gstride, int nvalid) {
  constexpr int CPR = HD / 8;  // chunks per row
  for (int idx = threadIdx.x; idx < ROWS * CPR; idx += NT) {
    const int r = idx / CPR, ch = idx % CPR;
    const bool ok = r < nvalid;
    const bf16* src = g + (int64_t)(ok ? r : 0) * gstride + ch * 8;
    cp_async16(s + swz<RS>(r, ch * 8), src, ok);
  }
}

__device__ __forceinline__ bool visible(int i, int j, int P, int Tn, int W) {
  if (j < P) return true;
  const int jm = j - P;
  return jm < Tn && jm <= i && (i - jm) < W;
}

// 8 consecutive elements as floats (one 16-byte access for 16-bit types, two for fp32)
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&o)[8]) {
  if constexpr (sizeof(T) == 2) {
    load16<T>(p, o);
  } else {
    float a[4], b[4];
    load16<T>(p, a);
    load16<T>(p + 4, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) { o[i] = a[i]; o[4 + i] = b[i]; }
  }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&o)[8]) {
  if constexpr (sizeof(T) == 2) {
    store16<T>(p, o);
  } else {
    float a[4] = {o[0], o[1], o[2], o[3]}, b[4] = {o[4], o[5], o[6], o[7]};
    store16<T>(p, a);
    store16<T>(p + 4, b);
  }
}
__device__ __forceinline__ void load8f(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

// rotate 4 interleaved pairs at position pos (pair indices p0..p0+3); sgn = -1 inverts
__device__ __forceinline__ void rope8(float (&v)[8], const float* inv_freq, int p0, float pos, float sgn) {
  if (inv_freq == nullptr) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float sn, cs;
    sincosf(pos * inv_freq[p0 + q], &sn, &cs);
    sn *= sgn;
    const float a = v[2 * q], b = v[2 * q + 1];
    v[2 * q] = a * cs - b * sn;
    v[2 * q + 1] = a * sn + b * cs;
  }
}

// ------------------------------------------------------------------ pack
// qkv: [B, T, 3D] (row stride sr, batch stride sb); pkv: [Bp, P, 2D] contiguous.
// One work item = 8 consecutive head-dim elements of one (b, key row j, head h).
template <typename T>
__global__ void pack_kernel(const T* __restrict__ qkv, int64_t sb, int64_t sr, const T* __restrict__ pkv, int Bp,
                            const float* __restrict__ inv_freq, bf16* __restrict__ Q, bf16* __restrict__ K,
                            bf16* __restrict__ V, int B, int Tn, int P, int H, int HD, int pos0) {
  const int D = H * HD;
  const int cpr = HD / 8;
  const int64_t total = (int64_t)B * (P + Tn) * H * cpr;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % cpr);
    int64_t r = e / cpr;
    const int h = (int)(r % H);
    r /= H;
    const int j = (int)(r % (P + Tn));  // combined key row
    const int b = (int)(r / (P + Tn));
    const int col = h * HD + c * 8;
    const int64_t kidx = (((int64_t)b * H + h) * (P + Tn) + j) * HD + c * 8;
    float k[8], v[8];
    if (j < P) {
      const T* row = pkv + ((int64_t)(Bp == 1 ? 0 : b) * P + j) * 2 * D;
      load8<T>(row + col, k);
      load8<T>(row + D + col, v);
    } else {
      const T* row = qkv + (int64_t)b * sb + (int64_t)(j - P) * sr;
      float q[8];
      load8<T>(row + col, q);
      load8<T>(row + D + col, k);
      load8<T>(row + 2 * D + col, v);
      // the query at main position i = j - P has rope position P + i + pos0 = j + pos0
      // (pos0: the main rows' offset in a longer sequence, e.g. a context-parallel shard)
      rope8(q, inv_freq, c * 4, (float)(j + pos0), 1.f);
      store8<bf16>(Q + (((int64_t)b * H + h) * Tn + (j - P)) * HD + c * 8, q);
    }
    rope8(k, inv_freq, c * 4, (float)(j < P ? j : j + pos0), 1.f);
    store8<bf16>(K + kidx, k);
    store8<bf16>(V + kidx, v);
  }
}

// ---------------------------------------------------------------- unpack
// dQa [B,H,T,d], dKa/dVa [B,H,P+T,d] fp32 -> dqkv [B,T,3D], dpkv [Bp,P,2D]
template <typename T>
__global__ void unpack_kernel(const float* __restrict__ dQa, const float* __restrict__ dKa,
                              const float* __restrict__ dVa, const float* __restrict__ inv_freq, T* __restrict__ dqkv,
                              T* __restrict__ dpkv, int Bp, int B, int Tn, int P, int H, int HD, int pos0) {
  const int D = H * HD;
  const int cpr = HD / 8;
  const int64_t total_main = (int64_t)B * Tn * H * cpr;
  const int64_t total_pre = (int64_t)Bp * P * H * cpr;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total_main + total_pre;
       e += (int64_t)gridDim.x * blockDim.x) {
    if (e < total_main) {
      const int c = (int)(e % cpr);
      int64_t r = e / cpr;
      const int h = (int)(r % H);
      r /= H;
      const int t = (int)(r % Tn);
      const int b = (int)(r / Tn);
      const int j = P + t;
      const int64_t bh = (int64_t)b * H + h;
      float dq[8], dk[8], dv[8];
      load8f(dQa + (bh * Tn + t) * HD + c * 8, dq);
      load8f(dKa + (bh * (P + Tn) + j) * HD + c * 8, dk);
      load8f(dVa + (bh * (P + Tn) + j) * HD + c * 8, dv);
      // inverse rotation: R(-a) applied to the gradient of the rotated vector
      rope8(dq, inv_freq, c * 4, (float)(j + pos0), -1.f);
      rope8(dk, inv_freq, c * 4, (float)(j + pos0), -1.f);
      T* row = dqkv + ((int64_t)b * Tn + t) * 3 * D + h * HD + c * 8;
      store8<T>(row, dq);
      store8<T>(row + D, dk);
      store8<T>(row + 2 * D, dv);
    } else {
      const int64_t e2 = e - total_main;
      const int c = (int)(e2 % cpr);
      int64_t r = e2 / cpr;
      const int h = (int)(r % H);
      r /= H;
      const int j = (int)(r % P);
      const int bp = (int)(r / P);
      float kx[8] = {0, 0, 0, 0, 0, 0, 0, 0}, vx[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      const int b_lo = Bp == 1 ? 0 : bp, b_hi = Bp == 1 ? B : bp + 1;
      for (int b = b_lo; b < b_hi; ++b) {
        const int64_t base = (((int64_t)b * H + h) * (P + Tn) + j) * HD + c * 8;
        float dk[8], dv[8];
        load8f(dKa + base, dk);
        load8f(dVa + base, dv);
#pragma unroll
        for (int i = 0; i < 8; ++i) { kx[i] += dk[i]; vx[i] += dv[i]; }
      }
      rope8(kx, inv_freq, c * 4, (float)j, -1.f);
      T* row = dpkv + ((int64_t)bp * P + j) * 2 * D + h * HD + c * 8;
      store8<T>(row, kx);
      store8<T>(row + D, vx);
    }
  }
}

// --------------------------------------------------------------- forward
template <int HD, int MT>
struct FwdCfg {
  static constexpr int NW = 4;
  static constexpr int BM = NW * 16 * MT;
  static constexpr int BN = 64;
  static constexpr int RS = ((HD + 63) / 64) * 8;  // chunks per smem row
  static constexpr int SQ = BM * RS * 8;
  static constexpr int SK = BN * RS * 8;
  static constexpr size_t smem = (size_t)(SQ + 4 * SK) * sizeof(bf16);
};

template <int HD, int MT>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const bf16* __restrict__ Q, const bf16* __restrict__ K,
                                                       const bf16* __restrict__ V, bf16* __restrict__ O,
                                                       float* __restrict__ LSE, int H, int Tn, int P, int W,
                                                       float scale_log2) {
  using C = FwdCfg<HD, MT>;
  constexpr int BM = C::BM, BN = C::BN, RS = C::RS, KS = HD / 16, DT = HD / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sK = sQ + C::SQ;          // 2 buffers
  bf16* sV = sK + 2 * C::SK;      // 2 buffers
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int bh = blockIdx.y;
  const int m0 = blockIdx.x * BM;
  const int L = P + Tn;
  const bf16* Qb = Q + (int64_t)bh * Tn * HD;
  const bf16* Kb = K + (int64_t)bh * L * HD;
  const bf16* Vb = V + (int64_t)bh * L * HD;

  // key tiles to visit: the prefix tiles, then the window tiles
  const int m_last = min(m0 + BM, Tn) - 1;
  const int jm_lo = max(0, m0 - W + 1);
  const int pre_tiles = (P + BN - 1) / BN;
  const int t_lo = max(pre_tiles, (P + jm_lo) / BN);
  const int t_hi = (P + m_last) / BN;
  const int n_win = t_hi >= t_lo ? t_hi - t_lo + 1 : 0;
  const int n_tiles = pre_tiles + n_win;
  auto tile_of = [&](int it) { return it < pre_tiles ? it : t_lo + (it - pre_tiles); };

  load_tile<HD, RS, BM, 128>(sQ, Qb + (int64_t)m0 * HD, HD, Tn - m0);
  cp_async_commit();
  if (n_tiles > 0) {
    const int n0 = tile_of(0) * BN;
    load_tile<HD, RS, BN, 128>(sK, Kb + (int64_t)n0 * HD, HD, L - n0);
    load_tile<HD, RS, BN, 128>(sV, Vb + (int64_t)n0 * HD, HD, L - n0);
  }
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  uint32_t qf[MT][KS][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
      ldsm_x4(qf[mt][ks], sQ + swz<RS>(warp * 16 * MT + mt * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8));

  float o[MT][DT][4];
  float mrow[MT][2], lrow[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int dt = 0; dt < DT; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][dt][e] = 0.f;
    mrow[mt][0] = mrow[mt][1] = -INFINITY;
    lrow[mt][0] = lrow[mt][1] = 0.f;
  }

  for (int it = 0; it < n_tiles; ++it) {
    const int buf = it & 1;
    const int n0 = tile_of(it) * BN;
    if (it + 1 < n_tiles) {
      const int n1 = tile_of(it + 1) * BN;
      load_tile<HD, RS, BN, 128>(sK + (buf ^ 1) * C::SK, Kb + (int64_t)n1 * HD, HD, L - n1);
      load_tile<HD, RS, BN, 128>(sV + (buf ^ 1) * C::SK, Vb + (int64_t)n1 * HD, HD, L - n1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const bf16* cK = sK + buf * C::SK;
    const bf16* cV = sV + buf * C::SK;

    float s[MT][BN / 8][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t kf[4];
        ldsm_x4(kf, cK + swz<RS>(np * 16 + (lane & 7) + (lane >> 4) * 8, ks * 16 + ((lane >> 3) & 1) * 8));
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma16816(s[mt][2 * np], qf[mt][ks], kf[0], kf[1]);
          mma16816(s[mt][2 * np + 1], qf[mt][ks], kf[2], kf[3]);
        }
      }
    }
    // mask: needed unless every (row, key) of the tile is visible
    const bool full = (n0 + BN <= P) ||
                      (n0 >= P && n0 + BN <= L && (n0 + BN - 1 - P) <= m0 && (m0 + BM - 1) - (n0 - P) < W);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int rbase = m0 + warp * 16 * MT + mt * 16 + g;
#pragma unroll
      for (int nt = 0; nt < BN / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[mt][nt][e] * scale_log2;
          if (!full) {
            const int i = rbase + ((e >> 1) << 3);
            const int j = n0 + nt * 8 + 2 * tq + (e & 1);
            if (!visible(i, j, P, Tn, W)) v = -INFINITY;
          }
          s[mt][nt][e] = v;
        }
      // online softmax for the two rows (g, g+8) this thread holds
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < BN / 8; ++nt) mx = fmaxf(mx, fmaxf(s[mt][nt][2 * r], s[mt][nt][2 * r + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mnew = fmaxf(mrow[mt][r], mx);
        const float muse = mnew == -INFINITY ? 0.f : mnew;
        const float corr = exp2f(mrow[mt][r] - muse);
        mrow[mt][r] = mnew;
        float ls = 0.f;
#pragma unroll
        for (int nt = 0; nt < BN / 8; ++nt) {
          const float p0 = exp2f(s[mt][nt][2 * r] - muse);
          const float p1 = exp2f(s[mt][nt][2 * r + 1] - muse);
          s[mt][nt][2 * r] = p0;
          s[mt][nt][2 * r + 1] = p1;
          ls += p0 + p1;
        }
        lrow[mt][r] = lrow[mt][r] * corr + ls;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt) {
          o[mt][dt][2 * r] *= corr;
          o[mt][dt][2 * r + 1] *= corr;
        }
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        pa[mt][0] = pack_bf16(s[mt][2 * kk][0], s[mt][2 * kk][1]);
        pa[mt][1] = pack_bf16(s[mt][2 * kk][2], s[mt][2 * kk][3]);
        pa[mt][2] = pack_bf16(s[mt][2 * kk + 1][0], s[mt][2 * kk + 1][1]);
        pa[mt][3] = pack_bf16(s[mt][2 * kk + 1][2], s[mt][2 * kk + 1][3]);
      }
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t vf[4];
        ldsm_x4_t(vf, cV + swz<RS>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma16816(o[mt][2 * dp], pa[mt], vf[0], vf[1]);
          mma16816(o[mt][2 * dp + 1], pa[mt], vf[2], vf[3]);
        }
      }
    }
    __syncthreads();
  }

  // finalize
  const int H_ = H;
  const int b = bh / H_, h = bh % H_;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float l = lrow[mt][r];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int i = m0 + warp * 16 * MT + mt * 16 + g + r * 8;
      if (i < Tn) {
        bf16* orow = O + (((int64_t)b * Tn + i) * H_ + h) * HD;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
          *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * tq) =
              pack_bf16(o[mt][dt][2 * r] * inv, o[mt][dt][2 * r + 1] * inv);
        if (tq == 0) LSE[(int64_t)bh * Tn + i] = (mrow[mt][r] + log2f(l)) * 0.69314718055994531f;
      }
    }
}

// ------------------------------------------------------------ backward pre
// Dd[bh, i] = sum_d dO[b,i,h,d] * O[b,i,h,d]; also converts LSE to log2 units.
// A group of HD/8 consecutive threads handles one row with 16-byte loads.
__global__ void bwd_pre_kernel(const bf16* __restrict__ dO, const bf16* __restrict__ O, const float* __restrict__ LSE,
                               float* __restrict__ Dd, float* __restrict__ LSE2, int B, int H, int Tn, int HD) {
  const int cpr = HD / 8;  // 4, 8, 12 or 16 threads per row
  const int64_t rows = (int64_t)B * H * Tn;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // every thread runs the same number of steps so the shuffles below stay convergent
  const int64_t nsteps = (rows * cpr + stride - 1) / stride;
  for (int64_t s = 0; s < nsteps; ++s) {
    const int64_t e = tid + s * stride;
    const int64_t r = e / cpr;
    const int c = (int)(e % cpr);
    float acc = 0.f;
    if (r < rows) {
      const int i = (int)(r % Tn);
      const int64_t bh = r / Tn;
      const int b = (int)(bh / H), h = (int)(bh % H);
      const int64_t off = (((int64_t)b * Tn + i) * H + h) * HD + c * 8;
      float a[8], o[8];
      load16<bf16>(dO + off, a);
      load16<bf16>(O + off, o);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += a[k] * o[k];
    }
    if ((32 % cpr) == 0) {  // a row's group lies inside one warp
      for (int o2 = 1; o2 < cpr; o2 <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
      if (r < rows && c == 0) {
        Dd[r] = acc;
        LSE2[r] = LSE[r] * 1.4426950408889634f;
      }
    } else if (r < rows) {  // head_dim 96: groups of 12 straddle warps
      atomicAdd(Dd + r, acc);
      if (c == 0) LSE2[r] = LSE[r] * 1.4426950408889634f;
    }
  }
}

// --------------------------------------------------------------- backward
template <int HD>
struct BwdCfg {
  static constexpr int BN = 64;                  // keys per CTA (4 warps x 16)
  static constexpr int BQ = HD <= 96 ? 64 : 32;  // queries per step
  static constexpr int RS = ((HD + 63) / 64) * 8;
  static constexpr int RSS = 8;                   // dS tile: 64 x (<=64) bf16
  static constexpr int SK = BN * RS * 8;
  static constexpr int SQ = BQ * RS * 8;
  static constexpr int SS = BN * RSS * 8;
  static constexpr size_t smem = (size_t)(2 * SK + 2 * SQ + SS) * sizeof(bf16) + 2 * BQ * sizeof(float);
  static constexpr int QB_PER_SPLIT = 16;
};

template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_kernel(
    const bf16* __restrict__ Q, const bf16* __restrict__ K, const bf16* __restrict__ V, const bf16* __restrict__ dO,
    const float* __restrict__ LSE2, const float* __restrict__ Dd, float* __restrict__ dQa, float* __restrict__ dKa,
    float* __restrict__ dVa, int H, int Tn, int P, int W, float scale, float scale_log2, int splits) {
  using C = BwdCfg<HD>;
  constexpr int BN = C::BN, BQ = C::BQ, RS = C::RS, RSS = C::RSS, KS = HD / 16, DT = HD / 8, QT = BQ / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sK = reinterpret_cast<bf16*>(smem_raw);
  bf16* sV = sK + C::SK;
  bf16* sQ = sV + C::SK;
  bf16* sdO = sQ + C::SQ;
  bf16* sdS = sdO + C::SQ;
  float* sL = reinterpret_cast<float*>(sdS + C::SS);
  float* sD = sL + BQ;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int kt = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int n0 = kt * BN;
  const int L = P + Tn;
  if (n0 >= L) return;

  // query range that can see this key tile
  int q_lo, q_hi;
  if (n0 < P) {
    q_lo = 0;
    q_hi = Tn - 1;
  } else {
    const int jm_lo = n0 - P, jm_hi = min(n0 + BN, L) - 1 - P;
    q_lo = jm_lo;
    q_hi = min(Tn - 1, jm_hi + W - 1);
  }
  const int qb_lo = q_lo / BQ, qb_hi = q_hi / BQ;
  const int nqb = qb_hi - qb_lo + 1;
  const int nsp = min(splits, (nqb + C::QB_PER_SPLIT - 1) / C::QB_PER_SPLIT);
  if (sp >= nsp) return;
  const int per = (nqb + nsp - 1) / nsp;
  const int qs = qb_lo + sp * per, qe = min(qb_hi + 1, qs + per);
  if (qs >= qe) return;

  const bf16* Kb = K + (int64_t)bh * L * HD;
  const bf16* Vb = V + (int64_t)bh * L * HD;
  const bf16* Qb = Q + (int64_t)bh * Tn * HD;
  const int64_t ostride = (int64_t)H * HD;
  const bf16* dOb = dO + (int64_t)b * Tn * ostride + h * HD;

  load_tile<HD, RS, BN, 128>(sK, Kb + (int64_t)n0 * HD, HD, L - n0);
  load_tile<HD, RS, BN, 128>(sV, Vb + (int64_t)n0 * HD, HD, L - n0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  uint32_t kf[KS][4], vf[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    ldsm_x4(kf[ks], sK + swz<RS>(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8));
    ldsm_x4(vf[ks], sV + swz<RS>(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8));
  }
  float dk[DT][4], dv[DT][4];
#pragma unroll
  for (int dt = 0; dt < DT; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[dt][e] = dv[dt][e] = 0.f;

  const int jrow0 = n0 + warp * 16 + g;  // key rows held by this thread: jrow0, jrow0 + 8

  for (int qb = qs; qb < qe; ++qb) {
    const int i0 = qb * BQ;
    load_tile<HD, RS, BQ, 128>(sQ, Qb + (int64_t)i0 * HD, HD, Tn - i0);
    load_tile<HD, RS, BQ, 128>(sdO, dOb + (int64_t)i0 * ostride, ostride, Tn - i0);
    cp_async_commit();
    for (int x = threadIdx.x; x < BQ; x += 128) {
      const bool ok = i0 + x < Tn;
      sL[x] = ok ? LSE2[(int64_t)bh * Tn + i0 + x] : 0.f;
      sD[x] = ok ? Dd[(int64_t)bh * Tn + i0 + x] : 0.f;
    }
    cp_async_wait<0>();
    __syncthreads();

    // S^T = K Q^T  (rows: this warp's 16 keys, cols: BQ queries)
    float st[QT][4];
#pragma unroll
    for (int nt = 0; nt < QT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t qf[4];
        ldsm_x4(qf, sQ + swz<RS>(np * 16 + (lane & 7) + (lane >> 4) * 8, ks * 16 + ((lane >> 3) & 1) * 8));
        mma16816(st[2 * np], kf[ks], qf[0], qf[1]);
        mma16816(st[2 * np + 1], kf[ks], qf[2], qf[3]);
      }
    // P^T
#pragma unroll
    for (int nt = 0; nt < QT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = jrow0 + ((e >> 1) << 3);
        const int il = nt * 8 + 2 * tq + (e & 1);
        const int i = i0 + il;
        const bool ok = i < Tn && j < L && visible(i, j, P, Tn, W);
        st[nt][e] = ok ? exp2f(st[nt][e] * scale_log2 - sL[il]) : 0.f;
      }
    // dV += P^T dO
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4] = {pack_bf16(st[2 * kk][0], st[2 * kk][1]), pack_bf16(st[2 * kk][2], st[2 * kk][3]),
                        pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]),
                        pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3])};
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t of[4];
        ldsm_x4_t(of, sdO + swz<RS>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
        mma16816(dv[2 * dp], pa, of[0], of[1]);
        mma16816(dv[2 * dp + 1], pa, of[2], of[3]);
      }
    }
    // dP^T = V dO^T
    float dpt[QT][4];
#pragma unroll
    for (int nt = 0; nt < QT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) dpt[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t of[4];
        ldsm_x4(of, sdO + swz<RS>(np * 16 + (lane & 7) + (lane >> 4) * 8, ks * 16 + ((lane >> 3) & 1) * 8));
        mma16816(dpt[2 * np], vf[ks], of[0], of[1]);
        mma16816(dpt[2 * np + 1], vf[ks], of[2], of[3]);
      }
    // dS^T = P^T (dP^T - D)   (kept in st)
#pragma unroll
    for (int nt = 0; nt < QT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int il = nt * 8 + 2 * tq + (e & 1);
        st[nt][e] = st[nt][e] * (dpt[nt][e] - sD[il]);
      }
    // dK += dS^T Q ; stash dS^T (bf16) for dQ
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4] = {pack_bf16(st[2 * kk][0], st[2 * kk][1]), pack_bf16(st[2 * kk][2], st[2 * kk][3]),
                        pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]),
                        pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3])};
      const int r0 = warp * 16 + g;
      *reinterpret_cast<uint32_t*>(sdS + swz<RSS>(r0, kk * 16 + 2 * tq)) = pa[0];
      *reinterpret_cast<uint32_t*>(sdS + swz<RSS>(r0 + 8, kk * 16 + 2 * tq)) = pa[1];
      *reinterpret_cast<uint32_t*>(sdS + swz<RSS>(r0, kk * 16 + 8 + 2 * tq)) = pa[2];
      *reinterpret_cast<uint32_t*>(sdS + swz<RSS>(r0 + 8, kk * 16 + 8 + 2 * tq)) = pa[3];
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t qf[4];
        ldsm_x4_t(qf, sQ + swz<RS>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
        mma16816(dk[2 * dp], pa, qf[0], qf[1]);
        mma16816(dk[2 * dp + 1], pa, qf[2], qf[3]);
      }
    }
    __syncthreads();
    // dQ[BQ x HD] += dS[BQ x BN] K[BN x HD]; warps tile (BQ/16 row tiles) x (d splits)
    {
      constexpr int MTQ = BQ / 16;
      constexpr int DSPLIT = 4 / MTQ;
      constexpr int DW = HD / DSPLIT;  // d columns per warp
      const int mt = warp % MTQ, ds = warp / MTQ;
      float dq[DW / 8][4];
#pragma unroll
      for (int x = 0; x < DW / 8; ++x)
#pragma unroll
        for (int e = 0; e < 4; ++e) dq[x][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t af[4];
        // A = dS (rows queries) from the key-major dS^T tile via ldmatrix.trans
        ldsm_x4_t(af, sdS + swz<RSS>(kk * 16 + (lane & 7) + (lane >> 4) * 8, mt * 16 + ((lane >> 3) & 1) * 8));
#pragma unroll
        for (int dp = 0; dp < DW / 16; ++dp) {
          uint32_t kf2[4];
          ldsm_x4_t(kf2, sK + swz<RS>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                     ds * DW + dp * 16 + (lane >> 4) * 8));
          mma16816(dq[2 * dp], af, kf2[0], kf2[1]);
          mma16816(dq[2 * dp + 1], af, kf2[2], kf2[3]);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int i = i0 + mt * 16 + g + r * 8;
        if (i < Tn) {
          float* dst = dQa + ((int64_t)bh * Tn + i) * HD + ds * DW;
#pragma unroll
          for (int x = 0; x < DW / 8; ++x)
            red_add2(dst + x * 8 + 2 * tq, dq[x][2 * r] * scale, dq[x][2 * r + 1] * scale);
        }
      }
    }
    __syncthreads();
  }
  // flush dK (scaled) and dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int j = jrow0 + r * 8;
    if (j < L) {
      float* dkd = dKa + ((int64_t)bh * L + j) * HD;
      float* dvd = dVa + ((int64_t)bh * L + j) * HD;
#pragma unroll
      for (int dt = 0; dt < DT; ++dt) {
        red_add2(dkd + dt * 8 + 2 * tq, dk[dt][2 * r] * scale, dk[dt][2 * r + 1] * scale);
        red_add2(dvd + dt * 8 + 2 * tq, dv[dt][2 * r], dv[dt][2 * r + 1]);
      }
    }
  }
}

}  // namespace attn

using attn::bf16;

#define TB_HD_SWITCH(HDV, ...)                                 \
  switch (HDV) {                                               \
    case 32: { constexpr int HD = 32; __VA_ARGS__; break; }    \
    case 64: { constexpr int HD = 64; __VA_ARGS__; break; }    \
    case 96: { constexpr int HD = 96; __VA_ARGS__; break; }    \
    case 128: { constexpr int HD = 128; __VA_ARGS__; break; }  \
    default: TORCH_CHECK(false, "attention: head_dim must be 32, 64, 96 or 128, got ", HDV); \
  }

// qkv [B, T, 3D] (last dim contiguous); pkv [Bp, P, 2D] or undefined.
// returns {Q, K, V} packed bf16 with RoPE applied.
// pos0: rope position offset of the main rows (prefix rows keep positions 0..P-1)
std::vector<at::Tensor> attn_pack(const at::Tensor& qkv, const c10::optional<at::Tensor>& pkv_opt, int64_t H,
                                  const c10::optional<at::Tensor>& inv_freq, int64_t pos0) {
  TB_CHECK_CUDA(qkv);
  TB_CHECK_LASTDIM(qkv);
  const at::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), Tn = qkv.size(1), D3 = qkv.size(2);
  TORCH_CHECK(D3 % 3 == 0 && (D3 / 3) % H == 0, "attn_pack: bad qkv width");
  const int D = D3 / 3, HD = D / H;
  TORCH_CHECK(HD % 16 == 0, "attn_pack: head_dim must be a multiple of 16");
  at::Tensor pkv;
  int P = 0, Bp = 1;
  if (pkv_opt.has_value() && pkv_opt->defined() && pkv_opt->size(1) > 0) {
    pkv = pkv_opt->to(qkv.scalar_type()).contiguous();
    P = pkv.size(1);
    Bp = pkv.size(0);
    TORCH_CHECK(pkv.size(2) == 2 * D && (Bp == 1 || Bp == B), "attn_pack: bad prefix shape");
  }
  at::Tensor inv = (inv_freq.has_value() && inv_freq->defined()) ? inv_freq->to(at::kFloat).contiguous() : at::Tensor();
  auto opts = qkv.options().dtype(at::kBFloat16);
  at::Tensor Q = at::empty({B, H, Tn, HD}, opts);
  at::Tensor K = at::empty({B, H, P + Tn, HD}, opts);
  at::Tensor V = at::empty({B, H, P + Tn, HD}, opts);
  const int64_t total = (int64_t)B * (P + Tn) * H * (HD / 8);
  if (total == 0) return {Q, K, V};
  TORCH_CHECK(qkv.stride(1) % 8 == 0 && qkv.stride(0) % 8 == 0 && aligned16(qkv), "attn_pack: qkv alignment");
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  TB_DISPATCH_FLOAT(qkv.scalar_type(), "attn_pack", [&] {
    attn::pack_kernel<scalar_t><<<blocks, 256, 0, stream()>>>(
        (const scalar_t*)qkv.data_ptr(), qkv.stride(0), qkv.stride(1),
        P ? (const scalar_t*)pkv.data_ptr() : nullptr, Bp, inv.defined() ? inv.data_ptr<float>() : nullptr,
        (bf16*)Q.data_ptr(), (bf16*)K.data_ptr(), (bf16*)V.data_ptr(), B, Tn, P, (int)H, HD, (int)pos0);
  });
  check_launch("attn_pack");
  return {Q, K, V};
}

// returns {O [B, T, H, d] bf16, LSE [B, H, T] fp32}
std::vector<at::Tensor> attn_fwd_packed(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, int64_t window,
                                        double scale) {
  const at::cuda::CUDAGuard g(Q.device());
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && Q.is_contiguous() && K.is_contiguous() && V.is_contiguous(),
              "attn_fwd: packed bf16 inputs");
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), HD = Q.size(3);
  const int P = K.size(2) - Tn;
  at::Tensor O = at::empty({B, Tn, H, HD}, Q.options());
  at::Tensor LSE = at::empty({B, H, Tn}, Q.options().dtype(at::kFloat));
  if (B * H * Tn == 0) return {O, LSE};
  const float sl2 = (float)scale * 1.4426950408889634f;
  const int W = (int)std::min<int64_t>(window, 1 << 30);
  TB_HD_SWITCH(HD, {
    constexpr int MT = HD <= 64 ? 2 : 1;
    using C = attn::FwdCfg<HD, MT>;
    auto kern = attn::attn_fwd_kernel<HD, MT>;
    if (C::smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::smem);
    dim3 grid((Tn + C::BM - 1) / C::BM, B * H);
    kern<<<grid, 128, C::smem, stream()>>>((const bf16*)Q.data_ptr(), (const bf16*)K.data_ptr(),
                                           (const bf16*)V.data_ptr(), (bf16*)O.data_ptr(), LSE.data_ptr<float>(), H,
                                           Tn, P, W, sl2);
  });
  check_launch("attn_fwd");
  return {O, LSE};
}

// returns {dQa, dKa, dVa} fp32 accumulators in the packed layouts
std::vector<at::Tensor> attn_bwd_packed(const at::Tensor& dO_in, const at::Tensor& Q, const at::Tensor& K,
                                        const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE,
                                        int64_t window, double scale) {
  const at::cuda::CUDAGuard g(Q.device());
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), HD = Q.size(3);
  const int P = K.size(2) - Tn;
  at::Tensor dO = dO_in.to(at::kBFloat16).contiguous();
  TORCH_CHECK(dO.sizes() == O.sizes(), "attn_bwd: dO shape");
  auto f32 = Q.options().dtype(at::kFloat);
  at::Tensor dQa = at::zeros({B, H, Tn, HD}, f32);
  at::Tensor dKa = at::zeros({B, H, P + Tn, HD}, f32);
  at::Tensor dVa = at::zeros({B, H, P + Tn, HD}, f32);
  if (B * H * Tn == 0) return {dQa, dKa, dVa};
  at::Tensor Dd = (32 % (HD / 8) == 0) ? at::empty({B, H, Tn}, f32) : at::zeros({B, H, Tn}, f32);
  at::Tensor L2 = at::empty({B, H, Tn}, f32);
  {
    const int64_t work = (int64_t)B * H * Tn * (HD / 8);
    const int blocks = (int)std::min<int64_t>((work + 255) / 256, (int64_t)num_sms() * 16);
    attn::bwd_pre_kernel<<<blocks, 256, 0, stream()>>>((const bf16*)dO.data_ptr(), (const bf16*)O.data_ptr(),
                                                       LSE.data_ptr<float>(), Dd.data_ptr<float>(),
                                                       L2.data_ptr<float>(), B, H, Tn, HD);
    check_launch("attn_bwd_pre");
  }
  const float sl2 = (float)scale * 1.4426950408889634f;
  const int W = (int)std::min<int64_t>(window, 1 << 30);
  TB_HD_SWITCH(HD, {
    using C = attn::BwdCfg<HD>;
    auto kern = attn::attn_bwd_kernel<HD>;
    if (C::smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::smem);
    const int nkt = (P + Tn + C::BN - 1) / C::BN;
    // the longest query range (a prefix tile sees all T queries) sets the split count
    const int max_qb = (Tn + C::BQ - 1) / C::BQ + 1;
    const int splits = std::max(1, (max_qb + C::QB_PER_SPLIT - 1) / C::QB_PER_SPLIT);
    dim3 grid(nkt * splits, B * H);
    kern<<<grid, 128, C::smem, stream()>>>((const bf16*)Q.data_ptr(), (const bf16*)K.data_ptr(),
                                           (const bf16*)V.data_ptr(), (const bf16*)dO.data_ptr(),
                                           L2.data_ptr<float>(), Dd.data_ptr<float>(), dQa.data_ptr<float>(),
                                           dKa.data_ptr<float>(), dVa.data_ptr<float>(), H, Tn, P, W, (float)scale,
                                           sl2, splits);
  });
  check_launch("attn_bwd");
  return {dQa, dKa, dVa};
}

// returns {dqkv [B, T, 3D], dpkv [Bp, P, 2D] (empty when P == 0)}
std::vector<at::Tensor> attn_unpack(const at::Tensor& dQa, const at::Tensor& dKa, const at::Tensor& dVa,
                                    const c10::optional<at::Tensor>& inv_freq, int64_t Bp, at::ScalarType dtype,
                                    int64_t pos0) {
  const at::cuda::CUDAGuard g(dQa.device());
  const int B = dQa.size(0), H = dQa.size(1), Tn = dQa.size(2), HD = dQa.size(3);
  const int P = dKa.size(2) - Tn;
  const int D = H * HD;
  at::Tensor inv = (inv_freq.has_value() && inv_freq->defined()) ? inv_freq->to(at::kFloat).contiguous() : at::Tensor();
  auto opts = dQa.options().dtype(dtype);
  at::Tensor dqkv = at::empty({B, Tn, 3 * D}, opts);
  at::Tensor dpkv = at::empty({P ? Bp : 0, P, 2 * D}, opts);
  const int64_t total = (int64_t)B * Tn * H * (HD / 8) + (int64_t)(P ? Bp : 0) * P * H * (HD / 8);
  if (total == 0) return {dqkv, dpkv};
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  TB_DISPATCH_FLOAT(dtype, "attn_unpack", [&] {
    attn::unpack_kernel<scalar_t><<<blocks, 256, 0, stream()>>>(
        dQa.data_ptr<float>(), dKa.data_ptr<float>(), dVa.data_ptr<float>(),
        inv.defined() ? inv.data_ptr<float>() : nullptr, (scalar_t*)dqkv.data_ptr(),
        P ? (scalar_t*)dpkv.data_ptr() : nullptr, (int)Bp, B, Tn, P, H, HD, (int)pos0);
  });
  check_launch("attn_unpack");
  return {dqkv, dpkv};
}

}  // namespace tb
