// Chunked neural-memory scan (paper semantics) on the 5th-generation tensor
// cores: one CTA per memory walks every chunk of its sequence.
//
// Memory: a 2-layer MLP M(x) = W2 silu(W1 x), x in R^64, hidden 256, with
// fp32 weights and momenta in global memory (L2-resident; read and rewritten
// once per chunk), stored hidden-index-fastest: W1^T, S1^T, W2, S2, each
// [64][256], so the thread owning hidden unit j (its TMEM lane) and its warp
// neighbours touch consecutive words.  Per chunk of C = 64 tokens (k_t, v_t, q_t):
//
//   Z   = [k; q] W1^T                (M=128 rows: 64 keys then 64 queries, N=256, K=64)
//   H   = silu(Z)                    threads -> shared memory (bf16)
//   P   = H W2^T                     (M=128, N=64, K=256): key rows = M(k), query rows = y
//   dP  = 2 (P_k - v) / 64           threads; also c*k, d*k, c*dP, d*dP (c_t, d_t below)
//   dH  = [dP; 0] W2                 (M=128, N=256, K=64)
//   dZ  = dH (.) silu'(Z_k)          threads -> shared memory (bf16)
//   G1  = dZ^T [c*k | d*k]           (M=256 as two 128-row halves, N=128, K=64 tokens)
//   G2T = H_k^T [c*dP | d*dP]        (same)
//   W <- A W + b S - G_c,  S <- p S - G_d      (both layers; threads, fp32)
//
// where, with per-token gates theta_t, eta_t, alpha_t,
//   a_t = prod_{s>t}(1-alpha_s), A = prod_s(1-alpha_s), E_t = prod_{s<=t} eta_s,
//   p = E_C, b = sum_t a_t E_t, d_t = theta_t prod_{s>t} eta_s,
//   c_t = theta_t F_t, F_t = a_t + eta_{t+1} F_{t+1} (F_C = 1).
// This is the chunked parallel form of S_t = eta_t S_{t-1} - theta_t grad l_t(W_0),
// W_t = (1-alpha_t) W_{t-1} + S_t with l_t = mean_j (M(k_t)_j - v_tj)^2 (every
// gradient of a chunk taken at its start weights); the queries of a chunk read
// the memory before the chunk's update.
//
// Warps: 0..7 two warpgroups of element-wise threads (thread = TMEM lane = row;
// the warpgroups split the columns), 8 MMA issuer (single thread), 9 producer
// (TMA loads of k, q, v; the chunk coefficients, one chunk ahead).
// TMEM: Z [0,256), P [256,320), dH [256,512), G1 [0,256), G2T [256,512).
// Shared tiles are 128-byte swizzled; several are read both as K-major and as
// MN-major operands.  All waits are bounded; a timeout records an error code.
#include "tc_common.cuh"

namespace tb {
namespace attn_tc {
CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows);
}
at::Tensor& tc_error_word(const at::Device& dev);

namespace memscan {

using bf16 = __nv_bfloat16;
constexpr int D = 64, HH = 256, C = 64;
constexpr int OFF_X = 0;                  // [128][64] keys (rows 0-63), queries (64-127)
constexpr int OFF_V = OFF_X + 16384;      // [64][64] values
constexpr int OFF_W1 = OFF_V + 8192;      // [256][64] bf16 W1
constexpr int OFF_W2 = OFF_W1 + 32768;    // [256][64] bf16 W2^T
constexpr int OFF_H = OFF_W2 + 32768;     // [128][256] as 4 slabs of [128][64]; later dZ in rows 64-127
constexpr int OFF_AD = OFF_H + 65536;     // [128][64] dP (rows 64-127 zero)
constexpr int OFF_KC = OFF_AD + 16384;    // 2 slabs [64][64]: c*k, d*k
constexpr int OFF_PC = OFF_KC + 16384;    // 2 slabs [64][64]: c*dP, d*dP
constexpr int OFF_COEF = OFF_PC + 16384;  // 2 buffers x COEF_N floats
constexpr int COEF_N = 2 * C + 4;         // c[64], d[64], A, b, p, pad
constexpr int OFF_SCR = OFF_COEF + 2 * COEF_N * 4;  // gate scratch: 3 x 64 floats + a_t 64
constexpr int OFF_BAR = OFF_SCR + 4 * C * 4;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TZ = 0, TP = 256, TDH = 256, TG1 = 0, TG2 = 256, TM_COLS = 512;

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}
// byte offset of 16-byte chunk ch of row r in a [rows][64 bf16] 128-byte-swizzled slab
__device__ __forceinline__ int swz(int r, int ch) { return r * 128 + ((ch ^ (r & 7)) << 4); }

// 8 fp32 -> one swizzled 16-byte chunk
__device__ __forceinline__ void st_chunk(uint8_t* slab, int r, int ch, const float* f) {
  *reinterpret_cast<uint4*>(slab + swz(r, ch)) =
      make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}
__device__ __forceinline__ void ld_chunk(const uint8_t* slab, int r, int ch, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(slab + swz(r, ch));
  float2 a = unpack2(u.x), b = unpack2(u.y), c = unpack2(u.z), d = unpack2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__global__ void __launch_bounds__(320, 1)
    memory_scan_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmV, float* __restrict__ W1g, float* __restrict__ S1g,
                       float* __restrict__ W2g, float* __restrict__ S2g, const float* __restrict__ theta,
                       const float* __restrict__ eta, const float* __restrict__ alpha, bf16* __restrict__ Y,
                       int Tn, unsigned* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* bar_x_full = bars + 0;
  uint64_t* bar_x_empty = bars + 1;
  uint64_t* bar_coef_full = bars + 2;   // [2]
  uint64_t* bar_coef_empty = bars + 4;  // [2]
  uint64_t* bar_z = bars + 6;           // MMA -> threads
  uint64_t* bar_h = bars + 7;           // threads -> MMA
  uint64_t* bar_p = bars + 8;
  uint64_t* bar_ad = bars + 9;
  uint64_t* bar_dh = bars + 10;
  uint64_t* bar_dz = bars + 11;
  uint64_t* bar_g = bars + 12;
  uint64_t* bar_w = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x;
  const int nchunks = (Tn + C - 1) / C;
  const int64_t soff = (int64_t)n * HH * D;
  float* W1 = W1g + soff;
  float* S1 = S1g + soff;
  float* W2 = W2g + soff;
  float* S2 = S2g + soff;

  if (threadIdx.x == 0) {
    tc::mbar_init(bar_x_full, 1);
    tc::mbar_init(bar_x_empty, 256);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(bar_coef_full + s, 1);
      tc::mbar_init(bar_coef_empty + s, 256);
    }
    tc::mbar_init(bar_z, 1);
    tc::mbar_init(bar_h, 256);
    tc::mbar_init(bar_p, 1);
    tc::mbar_init(bar_ad, 256);
    tc::mbar_init(bar_dh, 1);
    tc::mbar_init(bar_dz, 256);
    tc::mbar_init(bar_g, 1);
    tc::mbar_init(bar_w, 256);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (threadIdx.x < 256) {
    // bf16 operand copies of the incoming weights (row j of W1 and of W2^T);
    // zero rows 64-127 of the dP operand
    const int j = threadIdx.x;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const float* src = (w == 0 ? W1 : W2) + j;
      uint8_t* dst = smem + (w == 0 ? OFF_W1 : OFF_W2);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = src[(ch * 8 + e) * HH];
        st_chunk(dst, j, ch, f);
      }
    }
    reinterpret_cast<uint4*>(smem + OFF_AD + 64 * 128)[j * 2] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(smem + OFF_AD + 64 * 128)[j * 2 + 1] = make_uint4(0, 0, 0, 0);
    tc::fence_proxy_async_smem();
  }
  if (warp == 8) {
    tc::tmem_alloc(tmem_slot, TM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ producer
    float* scr = reinterpret_cast<float*>(smem + OFF_SCR);
    int issued = 0;
    for (int g = 0; g < nchunks; ++g) {
      const int c0 = g * C;
      bool ok = true;
      if (lane == 0) {
        if (g > 0) ok = tc::mbar_wait(bar_x_empty, (g - 1) & 1, abort_flag, err);
        if (ok) {
          tc::mbar_expect_tx(bar_x_full, 16384 + 8192);
          tc::tma_load_3d(smem + OFF_X, &tmK, bar_x_full, 0, c0, n);
          tc::tma_load_3d(smem + OFF_X + 8192, &tmQ, bar_x_full, 0, c0, n);
          tc::tma_load_3d(smem + OFF_V, &tmV, bar_x_full, 0, c0, n);
          issued = g + 1;
        }
      }
      if (!__all_sync(0xffffffffu, ok)) break;
      const int s = g & 1;
      if (g >= 2) {
        ok = tc::mbar_wait(bar_coef_empty + s, ((g >> 1) - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      // gates of this chunk (past the end: theta 0, eta 1, alpha 0 = identity)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = lane + 32 * h, tt = c0 + t;
        const bool in = tt < Tn;
        const int64_t gi = (int64_t)n * Tn + tt;
        scr[t] = in ? theta[gi] : 0.f;
        scr[C + t] = in ? eta[gi] : 1.f;
        scr[2 * C + t] = in ? alpha[gi] : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        // the chunk's nv valid tokens only (a padded token would still add S to W)
        const int nv = min(C, Tn - c0);
        float* cf = reinterpret_cast<float*>(smem + OFF_COEF) + s * COEF_N;
        float* at = scr + 3 * C;
        float a = 1.f, gp = 1.f, F = 0.f;
        for (int t = C - 1; t >= nv; --t) cf[t] = cf[C + t] = 0.f;
        for (int t = nv - 1; t >= 0; --t) {
          // a, gp: products over valid s > t of (1 - alpha_s), eta_s
          F = a + (t < nv - 1 ? scr[C + t + 1] * F : 0.f);
          cf[t] = scr[t] * F;
          cf[C + t] = scr[t] * gp;
          at[t] = a;
          a *= 1.f - scr[2 * C + t];
          gp *= scr[C + t];
        }
        float E = 1.f, b = 0.f;
        for (int t = 0; t < nv; ++t) {
          E *= scr[C + t];
          b += at[t] * E;
        }
        cf[2 * C] = a;       // A
        cf[2 * C + 1] = b;   // b
        cf[2 * C + 2] = gp;  // p
        tc::mbar_arrive(bar_coef_full + s);
      }
      __syncwarp();
    }
    if (lane == 0 && *abort_flag && issued > 0) {
      volatile int keep_waiting = 0;  // let the last copies land before the CTA exits
      tc::mbar_wait(bar_x_full, (issued - 1) & 1, &keep_waiting, nullptr, 1ll << 27);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_z = tc::idesc_bf16_f32(128, HH, false, false);
      constexpr uint32_t id_p = tc::idesc_bf16_f32(128, D, false, true);
      constexpr uint32_t id_g = tc::idesc_bf16_f32(128, 128, true, true);
      const uint32_t aX = tc::smem_addr(smem + OFF_X), aW1 = tc::smem_addr(smem + OFF_W1);
      const uint32_t aW2 = tc::smem_addr(smem + OFF_W2), aH = tc::smem_addr(smem + OFF_H);
      const uint32_t aAD = tc::smem_addr(smem + OFF_AD), aKC = tc::smem_addr(smem + OFF_KC);
      const uint32_t aPC = tc::smem_addr(smem + OFF_PC);
      for (int g = 0; g < nchunks; ++g) {
        const uint32_t ph = g & 1;
        if (g > 0 && !tc::mbar_wait(bar_w, ph ^ 1, abort_flag, err)) break;
        if (!tc::mbar_wait(bar_x_full, ph, abort_flag, err)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::umma_bf16(tmem + TZ, tc::sdesc_sw128(aX + 32 * kk, 16, 1024), tc::sdesc_sw128(aW1 + 32 * kk, 16, 1024),
                        id_z, kk > 0);
        tc::umma_commit(bar_z);
        if (!tc::mbar_wait(bar_h, ph, abort_flag, err)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HH / 16; ++kk)
          tc::umma_bf16(tmem + TP, tc::sdesc_sw128(aH + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                        tc::sdesc_sw128(aW2 + kk * 2048, 16384, 1024), id_p, kk > 0);
        tc::umma_commit(bar_p);
        if (!tc::mbar_wait(bar_ad, ph, abort_flag, err)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::umma_bf16(tmem + TDH, tc::sdesc_sw128(aAD + 32 * kk, 16, 1024),
                        tc::sdesc_sw128(aW2 + 32 * kk, 16, 1024), id_z, kk > 0);
        tc::umma_commit(bar_dh);
        if (!tc::mbar_wait(bar_dz, ph, abort_flag, err)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int kk = 0; kk < C / 16; ++kk) {
            // A: hidden rows [128h, 128h+128) x tokens, MN-major (two 64-hidden slabs, 16 KB apart)
            tc::umma_bf16(tmem + TG1 + h * 128,
                          tc::sdesc_sw128(aH + 2 * h * 16384 + 8192 + kk * 2048, 16384, 1024),
                          tc::sdesc_sw128(aKC + kk * 2048, 8192, 1024), id_g, kk > 0);
            tc::umma_bf16(tmem + TG2 + h * 128, tc::sdesc_sw128(aH + 2 * h * 16384 + kk * 2048, 16384, 1024),
                          tc::sdesc_sw128(aPC + kk * 2048, 8192, 1024), id_g, kk > 0);
          }
        }
        tc::umma_commit(bar_g);
      }
    }
  } else {
    // ------------------------------------------------------------ element-wise threads
    const int wg = warp >> 2;
    const int r = threadIdx.x & 127;  // TMEM lane / row
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float* coef = reinterpret_cast<const float*>(smem + OFF_COEF);
    for (int g = 0; g < nchunks; ++g) {
      const uint32_t ph = g & 1;
      const int c0 = g * C;
      // ---- H = silu(Z), this warpgroup's 128 hidden columns
      bool ok = tc::mbar_wait(bar_z, ph, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
#pragma unroll 1
      for (int pc = 0; pc < 4; ++pc) {
        const int col = wg * 128 + pc * 32;
        uint32_t z[32];
        tc::tmem_ld32(tl + TZ + col, z);
        tc::tmem_wait_ld();
        uint8_t* slab = smem + OFF_H + (col >> 6) * 16384;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = silu_(__uint_as_float(z[q * 8 + e]));
          st_chunk(slab, r, ((col & 63) >> 3) + q, f);
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_h);
      // ---- P: outputs (query rows) and the error terms (key rows), 32 columns per warpgroup
      ok = tc::mbar_wait(bar_p, ph, abort_flag, err) && tc::mbar_wait(bar_x_full, ph, abort_flag, err) &&
           tc::mbar_wait(bar_coef_full + (g & 1), (g >> 1) & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
      {
        const float* cf = coef + (g & 1) * COEF_N;
        uint32_t pv[32];
        tc::tmem_ld32(tl + TP + wg * 32, pv);
        tc::tmem_wait_ld();
        if (r >= C) {
          const int tt = c0 + r - C;
          if (tt < Tn) {
            uint4* dst = reinterpret_cast<uint4*>(Y + ((int64_t)n * Tn + tt) * D + wg * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dst[q] = make_uint4(pack2(__uint_as_float(pv[8 * q]), __uint_as_float(pv[8 * q + 1])),
                                  pack2(__uint_as_float(pv[8 * q + 2]), __uint_as_float(pv[8 * q + 3])),
                                  pack2(__uint_as_float(pv[8 * q + 4]), __uint_as_float(pv[8 * q + 5])),
                                  pack2(__uint_as_float(pv[8 * q + 6]), __uint_as_float(pv[8 * q + 7])));
          }
        } else {
          const float cr = cf[r], dr = cf[C + r];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int ch = wg * 4 + q;
            float vv[8], kv[8], dp[8], t0[8], t1[8];
            ld_chunk(smem + OFF_V, r, ch, vv);
            ld_chunk(smem + OFF_X, r, ch, kv);
#pragma unroll
            for (int e = 0; e < 8; ++e) dp[e] = (__uint_as_float(pv[8 * q + e]) - vv[e]) * (2.f / D);
            st_chunk(smem + OFF_AD, r, ch, dp);
#pragma unroll
            for (int e = 0; e < 8; ++e) { t0[e] = cr * dp[e]; t1[e] = dr * dp[e]; }
            st_chunk(smem + OFF_PC, r, ch, t0);
            st_chunk(smem + OFF_PC + 8192, r, ch, t1);
#pragma unroll
            for (int e = 0; e < 8; ++e) { t0[e] = cr * kv[e]; t1[e] = dr * kv[e]; }
            st_chunk(smem + OFF_KC, r, ch, t0);
            st_chunk(smem + OFF_KC + 8192, r, ch, t1);
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_ad);
      tc::mbar_arrive(bar_x_empty);
      // ---- dZ = dH (.) silu'(Z) for the key rows, into rows 64-127 of the H tile
      ok = tc::mbar_wait(bar_dh, ph, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
      if (r < C) {
#pragma unroll 1
        for (int pc = 0; pc < 4; ++pc) {
          const int col = wg * 128 + pc * 32;
          uint32_t z[32], dh[32];
          tc::tmem_ld32(tl + TZ + col, z);
          tc::tmem_ld32(tl + TDH + col, dh);
          tc::tmem_wait_ld();
          uint8_t* slab = smem + OFF_H + (col >> 6) * 16384;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              f[e] = __uint_as_float(dh[q * 8 + e]) * silu_grad_(__uint_as_float(z[q * 8 + e]));
            st_chunk(slab, C + r, ((col & 63) >> 3) + q, f);
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_dz);
      // ---- state update: thread = hidden row j of this warpgroup's half
      ok = tc::mbar_wait(bar_g, ph, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
      {
        const float* cf = coef + (g & 1) * COEF_N;
        const float A = cf[2 * C], b = cf[2 * C + 1], p = cf[2 * C + 2];
        const int j = wg * 128 + r;
#pragma unroll 1
        for (int layer = 0; layer < 2; ++layer) {
          float* Wl = (layer == 0 ? W1 : W2) + j;  // element i at Wl[i * HH]
          float* Sl = (layer == 0 ? S1 : S2) + j;
          uint8_t* op = smem + (layer == 0 ? OFF_W1 : OFF_W2);
          const uint32_t tg = tl + (layer == 0 ? TG1 : TG2) + wg * 128;
#pragma unroll 1
          for (int pc = 0; pc < 2; ++pc) {
            // the piece's 64 coalesced loads (a warp reads 32 consecutive words
            // each) are in flight while the gradient rows come out of TMEM
            float wv[32], sv[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              wv[e] = Wl[(pc * 32 + e) * HH];
              sv[e] = Sl[(pc * 32 + e) * HH];
            }
            uint32_t gc[32], gd[32];
            tc::tmem_ld32(tg + pc * 32, gc);
            tc::tmem_ld32(tg + 64 + pc * 32, gd);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float wn = A * wv[e] + b * sv[e] - __uint_as_float(gc[e]);
              sv[e] = p * sv[e] - __uint_as_float(gd[e]);
              wv[e] = wn;
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              Wl[(pc * 32 + e) * HH] = wv[e];
              Sl[(pc * 32 + e) * HH] = sv[e];
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) st_chunk(op, j, pc * 4 + q, wv + 8 * q);
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_w);
      tc::mbar_arrive(bar_coef_empty + (g & 1));
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 8) tc::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace memscan

// Paper-semantics memory scan for 2-layer memories of width 64, hidden 256,
// chunk 64.  W1t, S1t (first layer, transposed) and W2, S2: fp32
// [N, 64, 256] contiguous, updated in place.  k, v, q: bf16 [N, T, 64]
// contiguous; theta, eta, alpha: fp32 [N, T].  Returns y = M_{W_chunk}(q),
// bf16 [N, T, 64].
at::Tensor memory_scan_fwd(at::Tensor& W1, at::Tensor& S1, at::Tensor& W2T, at::Tensor& S2T, const at::Tensor& k,
                           const at::Tensor& v, const at::Tensor& q, const at::Tensor& theta, const at::Tensor& eta,
                           const at::Tensor& alpha) {
  using namespace memscan;
  const at::cuda::CUDAGuard guard(k.device());
  const int N = k.size(0), Tn = k.size(1);
  for (const at::Tensor* t : {&W1, &S1, &W2T, &S2T})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 3 &&
                    t->size(0) == N && t->size(1) == D && t->size(2) == HH,
                "memory_scan_fwd: states must be fp32 contiguous [N, 64, 256]");
  for (const at::Tensor* t : {&k, &v, &q})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 3 &&
                    t->size(0) == N && t->size(1) == Tn && t->size(2) == D && aligned16(*t),
                "memory_scan_fwd: k, v, q must be bf16 contiguous [N, T, 64]");
  for (const at::Tensor* t : {&theta, &eta, &alpha})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == (int64_t)N * Tn,
                "memory_scan_fwd: gates must be fp32 contiguous [N, T]");
  at::Tensor y = at::empty({N, Tn, D}, k.options());
  if ((int64_t)N * Tn == 0) return y;
  const CUtensorMap mk = attn_tc::make_map_3d(k.data_ptr(), D, Tn, N, C);
  const CUtensorMap mq = attn_tc::make_map_3d(q.data_ptr(), D, Tn, N, C);
  const CUtensorMap mv = attn_tc::make_map_3d(v.data_ptr(), D, Tn, N, C);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(memory_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set = true;
  }
  memory_scan_kernel<<<N, 320, SMEM_BYTES, stream()>>>(
      mk, mq, mv, W1.data_ptr<float>(), S1.data_ptr<float>(), W2T.data_ptr<float>(), S2T.data_ptr<float>(),
      theta.data_ptr<float>(), eta.data_ptr<float>(), alpha.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(), Tn,
      (unsigned*)tc_error_word(k.device()).data_ptr<int>());
  check_launch("memory_scan_fwd");
  return y;
}

}  // namespace tb
