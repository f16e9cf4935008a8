// Attention backward for head dim 96 on tcgen05 (the MAL configuration).
//
// The head-dim-64 backward (attention_tc.cu) keeps S^T, dP^T (128 columns
// each), dV, dK and a per-block dQ in tensor memory: with 96 columns per head
// that plan needs 544 of the 512 TMEM columns.  Here the work is split over
// two kernels, each of which fits:
//
//   dkdv96_kernel   key-major, persistent (the same work items, producer /
//                   MMA / two key-row warpgroups structure as the head-dim-64
//                   kernel): S^T = K Q^T, dP^T = V dO^T, P^T, dS^T in
//                   registers -> shared memory, dV += P^T dO, dK += dS^T Q.
//                   TMEM: S^T 128 + dP^T 128 + dV 96 + dK 96 = 448 columns.
//   dq_kernel<HD>   query-major: one CTA per (batch*head, 128-query tile)
//                   walks the key tiles its queries can see: S = Q K^T,
//                   dP = dO V^T, dS = P (dP - D) (thread = query row, two
//                   warpgroups split the 128 key columns) -> shared memory,
//                   dQ += dS K.  TMEM: S 128 + dP 128 + dQ HD.  dQ is
//                   written once per row (no atomic reduction); S and dP of
//                   the next key tile are issued as soon as the threads have
//                   read the current ones.
//
// The dQ kernel recomputes S and dP (7 products instead of 5), which buys the
// TMEM room and removes the red.global.add dQ traffic of the fused form.
//
// Tiles with 96 columns: columns 0-63 as 128-byte rows (128-byte swizzle),
// columns 64-95 right after them as 64-byte rows (64-byte swizzle) loaded by
// a second tensor map at x = 64 (the layout of the head-dim-96 forward).
// Products over the head dimension take 4 + 2 K-steps; products with the head
// dimension as N are an N = 64 and an N = 32 MMA.
// Every wait is bounded (error word, CTA unwinds); no multicast.
#include "tc_common.cuh"

#include <map>
#include <mutex>
#include <tuple>

namespace tb {

namespace attn_tc {
CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows,
                        uint32_t box_cols);
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();
}  // namespace attn_tc
namespace attn_tcb {
const at::Tensor& work_items(const at::Device& dev, int Tn, int P, int W);
}
at::Tensor& tc_error_word(const at::Device& dev);

namespace attn96 {

using bf16 = __nv_bfloat16;
constexpr int BQ = 128, BN = 128;                 // queries per block, keys per tile
constexpr int TILE_A = 128 * 64 * 2;              // 16 KB: 128 rows x columns 0-63
constexpr int TILE_B = 128 * 32 * 2;              // 8 KB: 128 rows x columns 64-95
constexpr int SLOT = TILE_A + TILE_B;             // one 96-column operand tile
constexpr int TILE_PS = 128 * 128 * 2;            // 32 KB: 128 x 128 bf16 (two 64-column blocks)
constexpr int QB_PER_SPLIT = 6;                   // must match attn_tcb's item list

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ unsigned range_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 32);
  if (hi <= lo) return 0u;
  const unsigned below_hi = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  return below_hi & ~((1u << lo) - 1u);
}

// K-major S-type product D = A B^T over the 96 head columns of two operand tiles
__device__ __forceinline__ void mma_hd96(uint32_t d, uint32_t aA, uint32_t aB, uint32_t idesc) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    tc::umma_bf16(d, tc::sdesc_sw128(aA + 32 * k, 16, 1024), tc::sdesc_sw128(aB + 32 * k, 16, 1024), idesc, k > 0);
#pragma unroll
  for (int k = 0; k < 2; ++k)
    tc::umma_bf16(d, tc::sdesc_sw64(aA + TILE_A + 32 * k, 16, 512), tc::sdesc_sw64(aB + TILE_A + 32 * k, 16, 512),
                  idesc, 1u);
}
// D (+)= A X with A a 128 x 128 K-major bf16 tile (two 64-column blocks) and X
// a 96-column operand tile read MN-major (its rows are the K dimension):
// columns 0-63 into d, 64-95 into d + 64
__device__ __forceinline__ void mma_x96(uint32_t d, uint32_t aA, uint32_t aX, bool acc0) {
  constexpr uint32_t id64 = tc::idesc_bf16_f32(128, 64, false, true);
  constexpr uint32_t id32 = tc::idesc_bf16_f32(128, 32, false, true);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t koff = (k >> 2) * (128 * 128) + (k & 3) * 32;
    const uint64_t ad = tc::sdesc_sw128(aA + koff, 16, 1024);
    const uint32_t acc = (acc0 || k > 0) ? 1u : 0u;
    tc::umma_bf16(d, ad, tc::sdesc_sw128(aX + k * 2048, 128 * 128, 1024), id64, acc);
    tc::umma_bf16(d + 64, ad, tc::sdesc_sw64(aX + TILE_A + k * 1024, 128 * 64, 512), id32, acc);
  }
}
// a row's 32 packed-bf16 words (64 columns) into a 128 x 128 K-major tile at column block cb
__device__ __forceinline__ void store_row64(uint8_t* tile, int cb, int r, const uint32_t (&w)[32]) {
  uint8_t* blk = tile + cb * (128 * 128) + r * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<uint4*>(blk + ((q ^ (r & 7)) << 4)) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// ------------------------------------------------------------------ pre-pass
// D[bh, i] = sum_d dO * O, lse2 = LSE * log2(e) ([BH][Tpad], zero padded), and
// zeroed dK / dV rows of key tiles split over several work items.
// 4 threads per row, 24 columns each.
__global__ void pre96_kernel(const bf16* __restrict__ dO, const bf16* __restrict__ O, const float* __restrict__ LSE,
                             float* __restrict__ Dd, float* __restrict__ L2, float* __restrict__ dKa,
                             float* __restrict__ dVa, int B, int H, int Tn, int Tpad, int P, int W, int RP) {
  constexpr int HD = 96;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r = e >> 2;
  const int c = (int)(e & 3);
  const int64_t bh = r / RP;
  const int i = (int)(r - bh * RP);
  const bool live = bh < (int64_t)B * H;
  float acc = 0.f;
  if (live && i < Tn) {
    const int b = (int)(bh / H), h = (int)(bh % H);
    const int64_t off = (((int64_t)b * Tn + i) * H + h) * HD + c * 24;
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      float a[8], o[8];
      load16<bf16>(dO + off + 8 * v, a);
      load16<bf16>(O + off + 8 * v, o);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += a[k] * o[k];
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  if (!live) return;
  if (i < Tpad && c == 0) {
    Dd[bh * Tpad + i] = acc;
    L2[bh * Tpad + i] = i < Tn ? LSE[bh * Tn + i] * 1.4426950408889634f : 0.f;
  }
  if (i < P + Tn) {
    // the key tile's query-block range, as the work-item list splits it
    const int n0 = i / BN * BN;
    int q_lo, q_hi;
    if (n0 < P) {
      q_lo = 0;
      q_hi = Tn - 1;
    } else {
      const int last_key = (n0 + BN < P + Tn ? n0 + BN : P + Tn) - 1 - P;
      q_lo = n0 - P;
      q_hi = last_key + W - 1 < Tn - 1 ? last_key + W - 1 : Tn - 1;
    }
    if (q_hi / BQ - q_lo / BQ + 1 > QB_PER_SPLIT) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const int64_t off = (bh * (P + Tn) + i) * HD + c * 24;
#pragma unroll
      for (int v = 0; v < 6; ++v) {
        reinterpret_cast<float4*>(dKa + off)[v] = z;
        reinterpret_cast<float4*>(dVa + off)[v] = z;
      }
    }
  }
}

// ------------------------------------------------------------------ dK / dV (key-major)
constexpr int K_OFF_K = 0, K_OFF_V = SLOT, K_OFF_Q = 2 * SLOT, K_OFF_DO = 4 * SLOT, K_OFF_PT = 6 * SLOT,
              K_OFF_DST = K_OFF_PT + TILE_PS, K_OFF_L = K_OFF_DST + TILE_PS, K_OFF_D = K_OFF_L + 2 * BQ * 4,
              K_OFF_BAR = K_OFF_D + 2 * BQ * 4;
constexpr int K_SMEM = K_OFF_BAR + 256 + 1024;
constexpr uint32_t TM_ST = 0, TM_DPT = 128, TM_DV = 256, TM_DK = 352;

struct Cursor {
  const int4* items;
  int n_pat, n_items, step;
  int i, it, j, nq, qs, n0, bh, split;
  __device__ Cursor(const int4* items_, int n_pat_, int n_items_)
      : items(items_), n_pat(n_pat_), n_items(n_items_), step(gridDim.x), i(blockIdx.x), it(0), j(0) {
    load();
  }
  __device__ void load() {
    if (i < n_items) {
      bh = i / n_pat;
      const int4 w = items[i - bh * n_pat];
      n0 = w.x * BN;
      qs = w.y;
      nq = w.z;
      split = w.w;
    }
  }
  __device__ bool valid() const { return i < n_items; }
  __device__ void next() {
    if (++j == nq) {
      j = 0;
      i += step;
      ++it;
      load();
    }
  }
};

__global__ void __launch_bounds__(320, 1)
    dkdv96_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmK2,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmV2,
                  const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQ2,
                  const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDO2,
                  const int4* __restrict__ items, int n_pat, int n_items, const float* __restrict__ L2,
                  const float* __restrict__ Dd, float* __restrict__ dKa, float* __restrict__ dVa, int H, int Tn,
                  int Tpad, int P, int W, float scale, float scale_log2, unsigned* __restrict__ err) {
  constexpr int HD = 96;
  if ((int)blockIdx.x >= n_items) return;
  const int L = P + Tn;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K_OFF_BAR);
  uint64_t* bar_kv_full = bars + 0;   // K/V of the item loaded (one slot)
  uint64_t* bar_kv_empty = bars + 1;  // the item's S^T/dP^T products are done with K/V
  uint64_t* bar_q_full = bars + 2;    // [2]
  uint64_t* bar_q_empty = bars + 4;   // [2]
  uint64_t* bar_s_full = bars + 6;
  uint64_t* bar_s_free = bars + 7;
  uint64_t* bar_p_full = bars + 8;
  uint64_t* bar_mma_done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tc::mbar_init(bar_kv_full, 1);
    tc::mbar_init(bar_kv_empty, 1);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(bar_q_full + s, 1);
      tc::mbar_init(bar_q_empty + s, 1);
    }
    tc::mbar_init(bar_s_full, 1);
    tc::mbar_init(bar_s_free, 256);
    tc::mbar_init(bar_p_full, 256);
    tc::mbar_init(bar_mma_done, 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      Cursor cur(items, n_pat, n_items);
      int g = 0, kv_issued = 0;
      while (cur.valid()) {
        if (cur.j == 0) {
          if (cur.it >= 1 && !tc::mbar_wait(bar_kv_empty, (cur.it - 1) & 1, abort_flag, err)) break;
          tc::mbar_expect_tx(bar_kv_full, 2 * SLOT);
          tc::tma_load_3d(smem + K_OFF_K, &tmK, bar_kv_full, 0, cur.n0, cur.bh);
          tc::tma_load_3d(smem + K_OFF_K + TILE_A, &tmK2, bar_kv_full, 64, cur.n0, cur.bh);
          tc::tma_load_3d(smem + K_OFF_V, &tmV, bar_kv_full, 0, cur.n0, cur.bh);
          tc::tma_load_3d(smem + K_OFF_V + TILE_A, &tmV2, bar_kv_full, 64, cur.n0, cur.bh);
          ++kv_issued;
        }
        const int s = g & 1;
        if (g >= 2 && !tc::mbar_wait(bar_q_empty + s, ((g >> 1) - 1) & 1, abort_flag, err)) break;
        const int q0 = (cur.qs + cur.j) * BQ;
        const int b = cur.bh / H, h = cur.bh - b * H;
        tc::mbar_expect_tx(bar_q_full + s, 2 * SLOT + 2 * BQ * 4);
        tc::tma_load_3d(smem + K_OFF_Q + s * SLOT, &tmQ, bar_q_full + s, 0, q0, cur.bh);
        tc::tma_load_3d(smem + K_OFF_Q + s * SLOT + TILE_A, &tmQ2, bar_q_full + s, 64, q0, cur.bh);
        tc::tma_load_4d(smem + K_OFF_DO + s * SLOT, &tmDO, bar_q_full + s, 0, h, q0, b);
        tc::tma_load_4d(smem + K_OFF_DO + s * SLOT + TILE_A, &tmDO2, bar_q_full + s, 64, h, q0, b);
        tc::bulk_load(smem + K_OFF_L + s * BQ * 4, L2 + (int64_t)cur.bh * Tpad + q0, BQ * 4, bar_q_full + s);
        tc::bulk_load(smem + K_OFF_D + s * BQ * 4, Dd + (int64_t)cur.bh * Tpad + q0, BQ * 4, bar_q_full + s);
        ++g;
        cur.next();
      }
      if (*abort_flag) {
        volatile int keep_waiting = 0;
        if (kv_issued > 0) tc::mbar_wait(bar_kv_full, (kv_issued - 1) & 1, &keep_waiting, nullptr, 1ll << 27);
        for (int t = max(0, g - 2); t < g; ++t)
          tc::mbar_wait(bar_q_full + (t & 1), (t >> 1) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t aK = tc::smem_addr(smem + K_OFF_K), aV = tc::smem_addr(smem + K_OFF_V);
      const uint32_t aPT = tc::smem_addr(smem + K_OFF_PT), aDST = tc::smem_addr(smem + K_OFF_DST);
      // K and V are read only by S^T and dP^T: the slot is released as soon as
      // the item's last S^T/dP^T products are done, so the next item's K/V load
      // while this item's last dV/dK products run
      auto issue_sdp = [&](const Cursor& c, int gg) -> bool {
        const int s = gg & 1;
        if (c.j == 0 && !tc::mbar_wait(bar_kv_full, c.it & 1, abort_flag, err)) return false;
        if (!tc::mbar_wait(bar_q_full + s, (gg >> 1) & 1, abort_flag, err)) return false;
        tc::tc_fence_after();
        const uint32_t aQ = tc::smem_addr(smem + K_OFF_Q + s * SLOT), aDO = tc::smem_addr(smem + K_OFF_DO + s * SLOT);
        mma_hd96(tmem + TM_ST, aK, aQ, id_s);
        mma_hd96(tmem + TM_DPT, aV, aDO, id_s);
        tc::umma_commit(bar_s_full);
        if (c.j == c.nq - 1) tc::umma_commit(bar_kv_empty);
        return true;
      };
      Cursor cur(items, n_pat, n_items);
      bool ok = issue_sdp(cur, 0);
      for (int g = 0; ok && cur.valid(); ++g) {
        if (!tc::mbar_wait(bar_s_free, g & 1, abort_flag, err)) break;
        tc::tc_fence_after();
        Cursor nxt = cur;
        nxt.next();
        if (nxt.valid() && !issue_sdp(nxt, g + 1)) break;
        if (!tc::mbar_wait(bar_p_full, g & 1, abort_flag, err)) break;
        tc::tc_fence_after();
        const int s = g & 1;
        const uint32_t aQ = tc::smem_addr(smem + K_OFF_Q + s * SLOT), aDO = tc::smem_addr(smem + K_OFF_DO + s * SLOT);
        mma_x96(tmem + TM_DV, aPT, aDO, cur.j > 0);
        mma_x96(tmem + TM_DK, aDST, aQ, cur.j > 0);
        tc::umma_commit(bar_mma_done);
        tc::umma_commit(bar_q_empty + s);
        cur = nxt;
      }
    }
  } else {
    // ------------------------------------------------------------ key-row threads
    const int wg = warp >> 2;
    const int r = threadIdx.x & 127;  // key row within the tile == TMEM lane
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    uint8_t* sPT = smem + K_OFF_PT;
    uint8_t* sDST = smem + K_OFF_DST;
    Cursor cur(items, n_pat, n_items);
    for (int g = 0; cur.valid(); ++g) {
      const int s = g & 1;
      const int q0 = (cur.qs + cur.j) * BQ;
      const int jk = cur.n0 + r;
      bool ok = tc::mbar_wait(bar_s_full, g & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
      int c_lo = 0, c_hi = 0;
      if (jk < P) {
        c_hi = min(BQ, Tn - q0);
      } else if (jk < L) {
        const int jm = jk - P;
        c_lo = min(BQ, max(0, jm - q0));
        c_hi = max(c_lo, min(BQ, min(Tn - 1, jm + W - 1) - q0 + 1));
      }
      const float* sl = reinterpret_cast<const float*>(smem + K_OFF_L + s * BQ * 4);
      const float* sd = reinterpret_cast<const float*>(smem + K_OFF_D + s * BQ * 4);
      const bool row_full = c_lo == 0 && c_hi == BQ;
      uint32_t pp[32], dd[32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = wg * 2 + cc;
        if (!__any_sync(0xffffffffu, c_lo < c * 32 + 32 && c_hi > c * 32)) {
#pragma unroll
          for (int x = 0; x < 16; ++x) pp[cc * 16 + x] = dd[cc * 16 + x] = 0u;
          continue;
        }
        uint32_t st[32], dp[32];
        tc::tmem_ld32(tl + TM_ST + c * 32, st);
        tc::tmem_ld32(tl + TM_DPT + c * 32, dp);
        tc::tmem_wait_ld();
        const unsigned vm = row_full ? 0xffffffffu : range_bits(c_lo - c * 32, c_hi - c * 32);
#pragma unroll
        for (int x = 0; x < 32; x += 4) {
          const int c0 = c * 32 + x;
          const float4 l4 = *reinterpret_cast<const float4*>(sl + c0);
          const float4 d4 = *reinterpret_cast<const float4*>(sd + c0);
          float p[4] = {ex2(fmaf(__uint_as_float(st[x]), scale_log2, -l4.x)),
                        ex2(fmaf(__uint_as_float(st[x + 1]), scale_log2, -l4.y)),
                        ex2(fmaf(__uint_as_float(st[x + 2]), scale_log2, -l4.z)),
                        ex2(fmaf(__uint_as_float(st[x + 3]), scale_log2, -l4.w))};
          if (!row_full) {
#pragma unroll
            for (int e = 0; e < 4; ++e) p[e] = (vm >> (x + e)) & 1u ? p[e] : 0.f;
          }
          pp[cc * 16 + (x >> 1)] = pack2(p[0], p[1]);
          pp[cc * 16 + (x >> 1) + 1] = pack2(p[2], p[3]);
          dd[cc * 16 + (x >> 1)] =
              pack2(p[0] * (__uint_as_float(dp[x]) - d4.x), p[1] * (__uint_as_float(dp[x + 1]) - d4.y));
          dd[cc * 16 + (x >> 1) + 1] =
              pack2(p[2] * (__uint_as_float(dp[x + 2]) - d4.z), p[3] * (__uint_as_float(dp[x + 3]) - d4.w));
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(bar_s_free);
      if (cur.j > 0) {  // the previous block's dV/dK MMAs have read P^T/dS^T
        ok = tc::mbar_wait(bar_mma_done, (g - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc::tc_fence_after();
      }
      store_row64(sPT, wg, r, pp);
      store_row64(sDST, wg, r, dd);
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_p_full);
      if (cur.j == cur.nq - 1) {
        // last block of the item: dK (scaled, warpgroup 0) and dV (warpgroup 1) rows
        ok = tc::mbar_wait(bar_mma_done, g & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc::tc_fence_after();
        float* base = wg == 0 ? dKa : dVa;
        const float mul = wg == 0 ? scale : 1.f;
#pragma unroll
        for (int hh = 0; hh < HD / 32; ++hh) {
          uint32_t v[32];
          tc::tmem_ld32(tl + (wg == 0 ? TM_DK : TM_DV) + hh * 32, v);
          tc::tmem_wait_ld();
          if (jk < L) {
            float* dst = base + ((int64_t)cur.bh * L + jk) * HD + hh * 32;
            if (cur.split) {
#pragma unroll
              for (int x = 0; x < 32; x += 4)
                tc::red_add4(dst + x, __uint_as_float(v[x]) * mul, __uint_as_float(v[x + 1]) * mul,
                             __uint_as_float(v[x + 2]) * mul, __uint_as_float(v[x + 3]) * mul);
            } else {
#pragma unroll
              for (int x = 0; x < 32; x += 4)
                *reinterpret_cast<float4*>(dst + x) =
                    make_float4(__uint_as_float(v[x]) * mul, __uint_as_float(v[x + 1]) * mul,
                                __uint_as_float(v[x + 2]) * mul, __uint_as_float(v[x + 3]) * mul);
            }
          }
        }
        tc::tc_fence_before();
      }
      cur.next();
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 9) tc::tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------ dQ (query-major)
constexpr int Q_OFF_Q = 0, Q_OFF_DO = SLOT, Q_OFF_K = 2 * SLOT, Q_OFF_V = 4 * SLOT, Q_OFF_DS = 6 * SLOT,
              Q_OFF_BAR = Q_OFF_DS + TILE_PS;
constexpr int Q_SMEM = Q_OFF_BAR + 256 + 1024;
constexpr uint32_t TQ_S = 0, TQ_DP = 128, TQ_DQ = 256;

__global__ void __launch_bounds__(320, 1)
    dq96_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmQ2,
                const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDO2,
                const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmK2,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmV2,
                const float* __restrict__ L2, const float* __restrict__ Dd, float* __restrict__ dQa, int H, int Tn,
                int Tpad, int P, int W, float scale, float scale_log2, unsigned* __restrict__ err) {
  constexpr int HD = 96;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q_OFF_BAR);
  uint64_t* bar_qd = bars + 0;        // Q and dO of the tile
  uint64_t* bar_kv_full = bars + 1;   // [2]
  uint64_t* bar_kv_empty = bars + 3;  // [2]
  uint64_t* bar_s_full = bars + 5;
  uint64_t* bar_s_free = bars + 6;
  uint64_t* bar_ds_full = bars + 7;
  uint64_t* bar_dq_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int q0 = blockIdx.x * BQ;
  const int b = bh / H, h = bh - b * H;

  // key tiles the tile's queries can see: the prefix tiles, then the window tiles
  const int q_last = min(q0 + BQ, Tn) - 1;
  const int jm_lo = max(0, q0 - W + 1);
  const int pre_tiles = (P + BN - 1) / BN;
  const int t_lo = max(pre_tiles, (P + jm_lo) / BN);
  const int t_hi = (P + q_last) / BN;
  const int n_tiles = pre_tiles + (t_hi >= t_lo ? t_hi - t_lo + 1 : 0);
  auto tile_n0 = [&](int it) { return (it < pre_tiles ? it : t_lo + (it - pre_tiles)) * BN; };

  if (threadIdx.x == 0) {
    tc::mbar_init(bar_qd, 1);
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(bar_kv_full + s, 1);
      tc::mbar_init(bar_kv_empty + s, 1);
    }
    tc::mbar_init(bar_s_full, 1);
    tc::mbar_init(bar_s_free, 256);
    tc::mbar_init(bar_ds_full, 256);
    tc::mbar_init(bar_dq_done, 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      tc::mbar_expect_tx(bar_qd, 2 * SLOT);
      tc::tma_load_3d(smem + Q_OFF_Q, &tmQ, bar_qd, 0, q0, bh);
      tc::tma_load_3d(smem + Q_OFF_Q + TILE_A, &tmQ2, bar_qd, 64, q0, bh);
      tc::tma_load_4d(smem + Q_OFF_DO, &tmDO, bar_qd, 0, h, q0, b);
      tc::tma_load_4d(smem + Q_OFF_DO + TILE_A, &tmDO2, bar_qd, 64, h, q0, b);
      int issued = 0;
      for (int it = 0; it < n_tiles; ++it) {
        const int s = it & 1;
        if (it >= 2 && !tc::mbar_wait(bar_kv_empty + s, ((it >> 1) - 1) & 1, abort_flag, err)) break;
        const int n0 = tile_n0(it);
        tc::mbar_expect_tx(bar_kv_full + s, 2 * SLOT);
        tc::tma_load_3d(smem + Q_OFF_K + s * SLOT, &tmK, bar_kv_full + s, 0, n0, bh);
        tc::tma_load_3d(smem + Q_OFF_K + s * SLOT + TILE_A, &tmK2, bar_kv_full + s, 64, n0, bh);
        tc::tma_load_3d(smem + Q_OFF_V + s * SLOT, &tmV, bar_kv_full + s, 0, n0, bh);
        tc::tma_load_3d(smem + Q_OFF_V + s * SLOT + TILE_A, &tmV2, bar_kv_full + s, 64, n0, bh);
        issued = it + 1;
      }
      if (*abort_flag) {
        volatile int keep_waiting = 0;
        tc::mbar_wait(bar_qd, 0, &keep_waiting, nullptr, 1ll << 27);
        for (int it = max(0, issued - 2); it < issued; ++it)
          tc::mbar_wait(bar_kv_full + (it & 1), (it >> 1) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t id_s = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t aQ = tc::smem_addr(smem + Q_OFF_Q), aDO = tc::smem_addr(smem + Q_OFF_DO);
      const uint32_t aDS = tc::smem_addr(smem + Q_OFF_DS);
      auto issue_sdp = [&](int it) -> bool {
        const int s = it & 1;
        if (!tc::mbar_wait(bar_kv_full + s, (it >> 1) & 1, abort_flag, err)) return false;
        tc::tc_fence_after();
        mma_hd96(tmem + TQ_S, aQ, tc::smem_addr(smem + Q_OFF_K + s * SLOT), id_s);
        mma_hd96(tmem + TQ_DP, aDO, tc::smem_addr(smem + Q_OFF_V + s * SLOT), id_s);
        tc::umma_commit(bar_s_full);
        return true;
      };
      bool ok = tc::mbar_wait(bar_qd, 0, abort_flag, err) && issue_sdp(0);
      for (int it = 0; ok && it < n_tiles; ++it) {
        if (!tc::mbar_wait(bar_s_free, it & 1, abort_flag, err)) break;  // threads have read S, dP
        tc::tc_fence_after();
        if (it + 1 < n_tiles && !issue_sdp(it + 1)) break;
        if (!tc::mbar_wait(bar_ds_full, it & 1, abort_flag, err)) break;
        tc::tc_fence_after();
        mma_x96(tmem + TQ_DQ, aDS, tc::smem_addr(smem + Q_OFF_K + (it & 1) * SLOT), it > 0);
        tc::umma_commit(bar_dq_done);
        tc::umma_commit(bar_kv_empty + (it & 1));
      }
    }
  } else {
    // ------------------------------------------------------------ query-row threads
    const int wg = warp >> 2;            // key columns [64 wg, 64 wg + 64) of every tile
    const int row = threadIdx.x & 127;   // query row == TMEM lane
    const int i = q0 + row;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    uint8_t* sDS = smem + Q_OFF_DS;
    const float lse2 = i < Tn ? L2[(int64_t)bh * Tpad + i] : 0.f;
    const float Dv = i < Tn ? Dd[(int64_t)bh * Tpad + i] : 0.f;
    const int win_lo = max(0, i - W + 1), win_hi = min(i, Tn - 1);  // visible main keys [win_lo, win_hi]
    bool ok = true;
    for (int it = 0; it < n_tiles; ++it) {
      const int n0 = tile_n0(it);
      ok = tc::mbar_wait(bar_s_full, it & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      // visible columns of this row: [0, pre_hi) prefix keys, [lo2, hi2) the window
      const int pre_hi = i < Tn ? min(BN, max(0, P - n0)) : 0;
      const int lo2 = max(pre_hi, P - n0 + win_lo);
      const int hi2 = i < Tn ? min(BN, P - n0 + win_hi + 1) : 0;
      uint32_t w[32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int a = (wg * 2 + cc) * 32;
        const unsigned vm = range_bits(-a, pre_hi - a) | range_bits(lo2 - a, hi2 - a);
        if (!__any_sync(0xffffffffu, vm != 0u)) {
#pragma unroll
          for (int x = 0; x < 16; ++x) w[cc * 16 + x] = 0u;
          continue;
        }
        uint32_t sr[32], dr[32];
        tc::tmem_ld32(tl + TQ_S + a, sr);
        tc::tmem_ld32(tl + TQ_DP + a, dr);
        tc::tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 32; x += 2) {
          float p0 = ex2(fmaf(__uint_as_float(sr[x]), scale_log2, -lse2));
          float p1 = ex2(fmaf(__uint_as_float(sr[x + 1]), scale_log2, -lse2));
          p0 = (vm >> x) & 1u ? p0 : 0.f;
          p1 = (vm >> (x + 1)) & 1u ? p1 : 0.f;
          w[cc * 16 + (x >> 1)] = pack2(p0 * (__uint_as_float(dr[x]) - Dv), p1 * (__uint_as_float(dr[x + 1]) - Dv));
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(bar_s_free);
      if (it > 0) {  // the previous tile's dQ MMA has read the dS buffer
        ok = tc::mbar_wait(bar_dq_done, (it - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
      }
      store_row64(sDS, wg, row, w);
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_ds_full);
    }
    if (ok && n_tiles > 0) {
      ok = tc::mbar_wait(bar_dq_done, (n_tiles - 1) & 1, abort_flag, err);
      if (__all_sync(0xffffffffu, ok)) {
        tc::tc_fence_after();
        // dQ = scale * sum dS K: warpgroup 0 columns 0-47, warpgroup 1 columns 48-95
        float* dst = dQa + ((int64_t)bh * Tn + i) * HD + wg * 48;
        uint32_t v[32], v2[16];
        tc::tmem_ld32(tl + TQ_DQ + wg * 48, v);
        tc::tmem_ld16(tl + TQ_DQ + wg * 48 + 32, v2);
        tc::tmem_wait_ld();
        if (i < Tn) {
#pragma unroll
          for (int x = 0; x < 32; x += 4)
            *reinterpret_cast<float4*>(dst + x) =
                make_float4(__uint_as_float(v[x]) * scale, __uint_as_float(v[x + 1]) * scale,
                            __uint_as_float(v[x + 2]) * scale, __uint_as_float(v[x + 3]) * scale);
#pragma unroll
          for (int x = 0; x < 16; x += 4)
            *reinterpret_cast<float4*>(dst + 32 + x) =
                make_float4(__uint_as_float(v2[x]) * scale, __uint_as_float(v2[x + 1]) * scale,
                            __uint_as_float(v2[x + 2]) * scale, __uint_as_float(v2[x + 3]) * scale);
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 9) tc::tmem_dealloc(tmem, 512);
}

// dO [B, T, H, HD] as a 4-D map (head dim, head, token, batch); box = cols x 1 x 128 x 1
CUtensorMap map_dO(const void* base, int B, int Tn, int H, uint32_t box_cols) {
  constexpr int HD = 96;
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)Tn, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)Tn * H * HD * 2};
  cuuint32_t box[4] = {box_cols, 1, (cuuint32_t)BQ, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = attn_tc::encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dO, head dim 96) failed: ", (int)r);
  return m;
}

}  // namespace attn96

// Head-dim-96 backward: same contract as attn_bwd_tc -> {dQa, dKa, dVa} fp32.
std::vector<at::Tensor> attn_bwd_tc96(const at::Tensor& dO_in, const at::Tensor& Q, const at::Tensor& K,
                                      const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE, int64_t window,
                                      double scale) {
  using namespace attn96;
  constexpr int HD = 96;
  const at::cuda::CUDAGuard g(Q.device());
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), hd = Q.size(3);
  TORCH_CHECK(hd == HD, "attn_bwd_tc96: head_dim must be 96");
  const int L = K.size(2), P = L - Tn;
  at::Tensor dO = dO_in.to(at::kBFloat16).contiguous();
  TORCH_CHECK(dO.sizes() == O.sizes() && aligned16(dO) && aligned16(Q) && aligned16(K) && aligned16(V) &&
                  Q.is_contiguous() && K.is_contiguous() && V.is_contiguous() && O.is_contiguous(),
              "attn_bwd_tc96: layout");
  auto f32 = Q.options().dtype(at::kFloat);
  at::Tensor dQa = at::empty({B, H, Tn, HD}, f32);
  at::Tensor dKa = at::empty({B, H, L, HD}, f32);
  at::Tensor dVa = at::empty({B, H, L, HD}, f32);
  if ((int64_t)B * H * Tn == 0) return {dQa.zero_(), dKa.zero_(), dVa.zero_()};
  const int W = (int)std::min<int64_t>(window, 1 << 30);
  const int Tpad = (Tn + BQ - 1) / BQ * BQ;
  const int nkt = (L + BN - 1) / BN;
  const int RP = std::max(Tpad, nkt * BN);
  at::Tensor Dd = at::empty({B, H, Tpad}, f32);
  at::Tensor L2 = at::empty({B, H, Tpad}, f32);
  {
    const int64_t work = (int64_t)B * H * RP * 4;
    pre96_kernel<<<(work + 255) / 256, 256, 0, stream()>>>(
        (const bf16*)dO.data_ptr(), (const bf16*)O.data_ptr(), LSE.data_ptr<float>(), Dd.data_ptr<float>(),
        L2.data_ptr<float>(), dKa.data_ptr<float>(), dVa.data_ptr<float>(), B, H, Tn, Tpad, P, W, RP);
    check_launch("attn_bwd_tc96 pre");
  }
  const CUtensorMap mk = attn_tc::make_map_3d(K.data_ptr(), HD, L, (uint64_t)B * H, BN, 64);
  const CUtensorMap mk2 = attn_tc::make_map_3d(K.data_ptr(), HD, L, (uint64_t)B * H, BN, 32);
  const CUtensorMap mv = attn_tc::make_map_3d(V.data_ptr(), HD, L, (uint64_t)B * H, BN, 64);
  const CUtensorMap mv2 = attn_tc::make_map_3d(V.data_ptr(), HD, L, (uint64_t)B * H, BN, 32);
  const CUtensorMap mq = attn_tc::make_map_3d(Q.data_ptr(), HD, Tn, (uint64_t)B * H, BQ, 64);
  const CUtensorMap mq2 = attn_tc::make_map_3d(Q.data_ptr(), HD, Tn, (uint64_t)B * H, BQ, 32);
  const CUtensorMap mdo = map_dO(dO.data_ptr(), B, Tn, H, 64);
  const CUtensorMap mdo2 = map_dO(dO.data_ptr(), B, Tn, H, 32);
  unsigned* err = (unsigned*)tc_error_word(Q.device()).data_ptr<int>();
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(dkdv96_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K_SMEM));
    C10_CUDA_CHECK(cudaFuncSetAttribute(dq96_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM));
    attr_set = true;
  }
  const float sl2 = (float)scale * 1.4426950408889634f;
  // dK, dV: key-major work items (the same list as the head-dim-64 backward)
  const at::Tensor& items = attn_tcb::work_items(Q.device(), Tn, P, W);
  const int n_pat = items.size(0);
  const int64_t n_items64 = (int64_t)n_pat * B * H;
  TORCH_CHECK(n_items64 < (1ll << 31), "attn_bwd_tc96: too many work items");
  const int n_items = (int)n_items64;
  dkdv96_kernel<<<std::min(n_items, num_sms()), 320, K_SMEM, stream()>>>(
      mk, mk2, mv, mv2, mq, mq2, mdo, mdo2, reinterpret_cast<const int4*>(items.data_ptr<int>()), n_pat, n_items,
      L2.data_ptr<float>(), Dd.data_ptr<float>(), dKa.data_ptr<float>(), dVa.data_ptr<float>(), H, Tn, Tpad, P, W,
      (float)scale, sl2, err);
  check_launch("attn_bwd_tc96 dkdv");
  // dQ: one CTA per (query tile, batch * head)
  dim3 grid((Tn + BQ - 1) / BQ, B * H);
  dq96_kernel<<<grid, 320, Q_SMEM, stream()>>>(mq, mq2, mdo, mdo2, mk, mk2, mv, mv2, L2.data_ptr<float>(),
                                               Dd.data_ptr<float>(), dQa.data_ptr<float>(), H, Tn, Tpad, P, W,
                                               (float)scale, sl2, err);
  check_launch("attn_bwd_tc96 dq");
  return {dQa, dKa, dVa};
}

}  // namespace tb
