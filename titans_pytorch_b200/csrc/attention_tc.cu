// Windowed causal attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), head_dim 64.
//
// One CTA = one (batch, head) and two query tiles of 128 rows (A and B) that
// share every K/V tile; 10 warps:
//   warp 8      TMA producer: both Q tiles once, then K/V tiles of 128 keys
//               through a 2-stage ring (128-byte swizzled, i.e. already in the
//               UMMA shared-memory layout)
//   warp 9      TMEM allocator + single-thread MMA issuer.  Per key tile j it
//               issues, in ping-pong order,
//                 O_A += P_A V_j ; S_A = Q_A K_{j+1}^T ; O_B += P_B V_j ; S_B = Q_B K_{j+1}^T
//               so the tensor core works on one tile while the softmax warps
//               of the other tile run.
//   warps 0..3  softmax of tile A, warps 4..7 softmax of tile B; thread r of a
//               warpgroup owns query row r = TMEM lane r: it reads its S row
//               with tcgen05.ld, applies scale + prefix/window mask (as column
//               ranges) + online max, writes P (bf16) to shared memory in the
//               UMMA K-major layout, rescales its O row in TMEM when the max
//               grew, and at the end normalises O and stores it.
//
// TMEM: S_A cols [0,128), S_B [128,256), O_A [256,320), O_B [320,384).
// Key tiles visited: tiles holding prefix keys, then the tiles intersecting the
// CTA's window, so work is O(T * (P + window)).  Every mbarrier wait is
// bounded; on a timeout the CTA records an error code and unwinds (TMEM is
// always released).
#include <map>
#include <mutex>
#include <tuple>

#include "tc_common.cuh"

namespace tb {
namespace attn_tc {

using bf16 = __nv_bfloat16;

constexpr int BM = 128;  // rows per query tile
constexpr int NQ = 2;    // query tiles per CTA
constexpr int BN = 128;  // keys per tile
constexpr int TILE_P = BM * BN * 2;

// Shared-memory layout for head dim HD (64 or 96).  A Q/K/V tile holds
// columns 0-63 as 128-byte rows (128-byte swizzle) and, for HD = 96, columns
// 64-95 right after them as 64-byte rows (64-byte swizzle): 24 KB per 128 rows
// instead of the 32 KB a padding to 128 columns would take, so two query
// tiles, two K/V stages and two P tiles still fit (208 KB).
template <int HD>
struct Fwd {
  static_assert(HD == 64 || HD == 96, "head_dim 64 or 96");
  static constexpr int NS = HD == 64 ? 3 : 2;  // K/V stages (three fit at head dim 64)
  static constexpr int TILE_QA = BM * 64 * 2, TILE_QB = HD > 64 ? BM * 32 * 2 : 0, TILE_Q = TILE_QA + TILE_QB;
  static constexpr int TILE_KA = BN * 64 * 2, TILE_KB = HD > 64 ? BN * 32 * 2 : 0, TILE_K = TILE_KA + TILE_KB;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NQ * TILE_Q;
  static constexpr int OFF_V = OFF_K + NS * TILE_K;
  static constexpr int OFF_P = OFF_V + NS * TILE_K;
  static constexpr int OFF_RED = OFF_P + NQ * TILE_P;  // [2 phases][NQ][2 halves][BM] fp32 row exchange
  static constexpr int OFF_BAR = OFF_RED + 2 * NQ * 2 * BM * 4;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
};
constexpr uint32_t TM_S = 0, TM_O = 256, TM_COLS = 512;
// warps 0-15: softmax (query tile = warp / 8, column half = (warp / 4) & 1); 16: producer; 17: MMA
constexpr int SOFTMAX_WARPS = 16, PRODUCER_WARP = 16, MMA_WARP = 17;
constexpr int NTHREADS = 32 * 18;

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Bits [lo, hi) of a 32-bit word (lo, hi clamped to [0, 32]): the visible
// columns of one 32-column chunk, so the per-element mask is one bit test.
__device__ __forceinline__ unsigned range_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 32);
  if (hi <= lo) return 0u;
  const unsigned below_hi = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  return below_hi & ~((1u << lo) - 1u);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes of work)
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2split(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for two values on the FMA pipe, to take part of the exponentials off
// the MUFU unit (16 results per clock per SM), as FlashAttention-4 (Dao et
// al., 2025) does.  Method: 2^x = 2^j * 2^f with j = rint(x) (the 1.5*2^23
// rounding add) and f = x - j in [-0.5, 0.5]; 2^f is a cubic whose
// coefficients were fitted here to minimise the relative error on that
// interval (max 1.1e-4, far below bf16's 3.9e-3 resolution of P); 2^j is added
// to the exponent field.  x < -125 gives 0 (masked scores are -inf).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  const float c0 = 0.99994105f, c1 = 0.69341969f, c2 = 0.24250251f, c3 = 0.054287549f;
  const float m = 12582912.f;  // 1.5 * 2^23
  const uint64_t xc = f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = fadd2(xc, f2(m, m));                       // rint(x) in the low mantissa bits
  const uint64_t f = ffma2(fadd2(t, f2(-m, -m)), f2(-1.f, -1.f), xc);  // x - rint(x)
  uint64_t p = ffma2(f, f2(c3, c3), f2(c2, c2));
  p = ffma2(p, f, f2(c1, c1));
  p = ffma2(p, f, f2(c0, c0));
  float p0, p1, t0, t1;
  f2split(p, p0, p1);
  f2split(t, t0, t1);
  y0 = x0 < -125.f ? 0.f : __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = x1 < -125.f ? 0.f : __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Test hook: y = exp2_poly2(x) elementwise (pairs), so the polynomial's error
// bound can be checked directly against exp2 on the device.
__global__ void exp2_poly_eval_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  const int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 < n) {
    exp2_poly2(x[i], x[i + 1], y[i], y[i + 1]);
  } else if (i < n) {
    float dummy;
    exp2_poly2(x[i], 0.f, y[i], dummy);
  }
}

// tmQ/tmK/tmV: columns 0-63 (128-byte swizzle); tmQb/tmKb/tmVb: columns 64-95
// (64-byte swizzle), used when HD = 96.
// 18 warps: two of the four schedulers hold 5 warps, so 96 registers per thread
// (5 x 32 x 96 <= 16,384 per scheduler)
template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQb,
                       const __grid_constant__ CUtensorMap tmKb, const __grid_constant__ CUtensorMap tmVb,
                       bf16* __restrict__ O, float* __restrict__ LSE,
                       int H, int Tn, int P, int W, float scale_log2, unsigned* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using C = Fwd<HD>;
  constexpr int NS = C::NS;
  constexpr bool kSplit = HD > 64;  // columns 64-95 in a second, 64-byte-swizzled tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kv_full = bars + 1;          // [NS]
  uint64_t* bar_kv_empty = bars + 1 + NS;    // [NS]
  uint64_t* bar_s_full = bars + 1 + 2 * NS;  // [NQ]
  uint64_t* bar_p_full = bars + 3 + 2 * NS;  // [NQ]
  uint64_t* bar_o_done = bars + 5 + 2 * NS;  // [NQ]
  uint64_t* bar_x = bars + 7 + 2 * NS;       // [NQ] row max / sum exchange between the two column halves
  uint64_t* bar_s_free = bars + 9 + 2 * NS;  // [NQ] the row threads have read S (the next S may be issued)
  static_assert(11 + 2 * NS <= 24, "forward barriers overlap the TMEM address word");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int m0 = blockIdx.x * (NQ * BM);
  const int L = P + Tn;

  // key tiles: prefix tiles, then the tiles intersecting the CTA's window
  const int m_last = min(m0 + NQ * BM, Tn) - 1;
  const int jm_lo = max(0, m0 - W + 1);
  const int pre_tiles = (P + BN - 1) / BN;
  const int t_lo = max(pre_tiles, (P + jm_lo) / BN);
  const int t_hi = (P + m_last) / BN;
  const int n_tiles = pre_tiles + (t_hi >= t_lo ? t_hi - t_lo + 1 : 0);
  auto tile_n0 = [&](int it) { return (it < pre_tiles ? it : t_lo + (it - pre_tiles)) * BN; };

  if (threadIdx.x == 0) {
    tc::mbar_init(bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_kv_full + s, 1);
      tc::mbar_init(bar_kv_empty + s, 1);
    }
    for (int q = 0; q < NQ; ++q) {
      tc::mbar_init(bar_s_full + q, 1);
      tc::mbar_init(bar_p_full + q, 256);
      tc::mbar_init(bar_o_done + q, 1);
      tc::mbar_init(bar_x + q, 256);
      tc::mbar_init(bar_s_free + q, 256);
    }
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == MMA_WARP) {
    tc::tmem_alloc(tmem_slot, TM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      tc::tma_prefetch_desc(&tmQ);
      tc::tma_prefetch_desc(&tmK);
      tc::tma_prefetch_desc(&tmV);
      tc::mbar_expect_tx(bar_q, NQ * C::TILE_Q);
      for (int q = 0; q < NQ; ++q) {
        tc::tma_load_3d(smem + C::OFF_Q + q * C::TILE_Q, &tmQ, bar_q, 0, m0 + q * BM, bh);
        if constexpr (kSplit)
          tc::tma_load_3d(smem + C::OFF_Q + q * C::TILE_Q + C::TILE_QA, &tmQb, bar_q, 64, m0 + q * BM, bh);
      }
      int issued = 0;
      for (int it = 0; it < n_tiles; ++it) {
        const int s = it % NS;
        if (it >= NS && !tc::mbar_wait(bar_kv_empty + s, ((it / NS) - 1) & 1, abort_flag, err)) break;
        const int n0 = tile_n0(it);
        tc::mbar_expect_tx(bar_kv_full + s, 2 * C::TILE_K);
        tc::tma_load_3d(smem + C::OFF_K + s * C::TILE_K, &tmK, bar_kv_full + s, 0, n0, bh);
        tc::tma_load_3d(smem + C::OFF_V + s * C::TILE_K, &tmV, bar_kv_full + s, 0, n0, bh);
        if constexpr (kSplit) {
          tc::tma_load_3d(smem + C::OFF_K + s * C::TILE_K + C::TILE_KA, &tmKb, bar_kv_full + s, 64, n0, bh);
          tc::tma_load_3d(smem + C::OFF_V + s * C::TILE_K + C::TILE_KA, &tmVb, bar_kv_full + s, 64, n0, bh);
        }
        issued = it + 1;
      }
      if (*abort_flag) {
        volatile int keep_waiting = 0;  // let issued copies land before exit (bounded)
        for (int it = max(0, issued - NS); it < issued; ++it)
          tc::mbar_wait(bar_kv_full + (it % NS), (it / NS) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_o = tc::idesc_bf16_f32(BM, 64, false, true);    // O columns 0-63
      constexpr uint32_t idesc_o2 = tc::idesc_bf16_f32(BM, 32, false, true);   // O columns 64-95 (HD = 96)
      bool ok = tc::mbar_wait(bar_q, 0, abort_flag, err);
      auto issue_s = [&](int q, int it) {
        const uint32_t aQ = tc::smem_addr(smem + C::OFF_Q + q * C::TILE_Q);
        const uint32_t aK = tc::smem_addr(smem + C::OFF_K + (it % NS) * C::TILE_K);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc::umma_bf16(tmem + TM_S + q * BN, tc::sdesc_sw128(aQ + 32 * k, 16, 1024),
                        tc::sdesc_sw128(aK + 32 * k, 16, 1024), idesc_s, k > 0);
        if constexpr (kSplit) {
#pragma unroll
          for (int k = 0; k < 2; ++k)
            tc::umma_bf16(tmem + TM_S + q * BN, tc::sdesc_sw64(aQ + C::TILE_QA + 32 * k, 16, 512),
                          tc::sdesc_sw64(aK + C::TILE_KA + 32 * k, 16, 512), idesc_s, 1u);
        }
        tc::umma_commit(bar_s_full + q);
      };
      if (ok) ok = tc::mbar_wait(bar_kv_full, 0, abort_flag, err);
      if (ok) {
        tc::tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      // Per key tile and query tile, head dim 64: the next tile's scores as soon
      // as the row threads have read this tile's (so S(it+1) runs while they
      // compute P(it)), then O += P V once P(it) is in shared memory.  Head dim
      // 96: O += P V first (its S is 1.5x longer, and the next P store waits for
      // this PV), then the next scores.
      constexpr bool kEarlyS = HD == 64;
      auto next_s = [&](int q, int it) -> bool {
        if (q == 0 && !tc::mbar_wait(bar_kv_full + ((it + 1) % NS), ((it + 1) / NS) & 1, abort_flag, err))
          return false;
        if (!tc::mbar_wait(bar_s_free + q, it & 1, abort_flag, err)) return false;
        tc::tc_fence_after();
        issue_s(q, it + 1);
        return true;
      };
      for (int it = 0; ok && it < n_tiles; ++it) {
        const int s = it % NS;
        const bool more = it + 1 < n_tiles;
        const uint32_t aV = tc::smem_addr(smem + C::OFF_V + s * C::TILE_K);
        for (int q = 0; q < NQ && ok; ++q) {
          if (kEarlyS && more && !next_s(q, it)) {
            ok = false;
            break;
          }
          if (!tc::mbar_wait(bar_p_full + q, it & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t aP = tc::smem_addr(smem + C::OFF_P + q * TILE_P);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint64_t ad = tc::sdesc_sw128(aP + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = tc::sdesc_sw128(aV + k * 2048, BN * 128, 1024);  // V: MN-major
            tc::umma_bf16(tmem + TM_O + q * HD, ad, bd, idesc_o, (it > 0 || k > 0) ? 1u : 0u);
            if constexpr (kSplit) {
              const uint64_t bd2 = tc::sdesc_sw64(aV + C::TILE_KA + k * 1024, BN * 64, 512);
              tc::umma_bf16(tmem + TM_O + q * HD + 64, ad, bd2, idesc_o2, (it > 0 || k > 0) ? 1u : 0u);
            }
          }
          tc::umma_commit(bar_o_done + q);
          if (q == NQ - 1) tc::umma_commit(bar_kv_empty + s);
          if (!kEarlyS && more && !next_s(q, it)) {
            ok = false;
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    // Two warpgroups per query tile, one per 64-column half of the 128 keys:
    // thread = (query row = TMEM lane, half).  The halves exchange their row
    // max every tile (and their row sums at the end) through shared memory,
    // synchronised by an mbarrier with a bounded wait; each half rescales and
    // stores its half of the O columns.  S is released as soon as it is in
    // registers, so the tensor core computes the next tile's scores meanwhile.
    constexpr int HO = HD / 2;            // O columns per half (32 or 48)
    const int q = warp >> 3;              // query tile of this warpgroup pair
    const int hf = (warp >> 2) & 1;       // column half
    const int row = threadIdx.x & 127;    // TMEM lane
    const int i = m0 + q * BM + row;      // query index
    const int c0 = hf * 64;               // first key column of this half
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t tS = tl + TM_S + q * BN + c0, tO = tl + TM_O + q * HD + hf * HO;
    uint8_t* sP = smem + C::OFF_P + q * TILE_P + hf * (BM * 128);  // this half's 64-column K-major block
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
    auto red_at = [&](int phase, int h) -> float* { return red + (((phase & 1) * NQ + q) * 2 + h) * BM + row; };
    // this thread's O half: one 32-column load plus, for HD = 96, one 16-column load
    auto o_load = [&](uint32_t (&r)[32], uint32_t (&r2)[16]) {
      tc::tmem_ld32(tO, r);
      if constexpr (HO > 32) tc::tmem_ld16(tO + 32, r2);
      tc::tmem_wait_ld();
    };
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    const int win_lo = max(0, i - W + 1), win_hi = min(i, Tn - 1);  // visible main keys [win_lo, win_hi]
    for (int it = 0; it < n_tiles; ++it) {
      const int n0 = tile_n0(it);
      ok = tc::mbar_wait(bar_s_full + q, it & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      float s[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(tS + c * 32, r);
#pragma unroll
        for (int x = 0; x < 32; ++x) s[c * 32 + x] = __uint_as_float(r[x]);
      }
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_s_free + q);  // S is in registers: the next tile's scores may be written
      // visible tile columns: [0, pre_hi) are prefix keys; [lo2, hi2) the window
      const int pre_hi = min(BN, max(0, P - n0));
      const int lo2 = max(pre_hi, P - n0 + win_lo);
      const int hi2 = min(BN, P - n0 + win_hi + 1);
      unsigned vm[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int a = c0 + c * 32;
        vm[c] = range_bits(-a, pre_hi - a) | range_bits(lo2 - a, hi2 - a);
      }
      const bool warp_full = __all_sync(0xffffffffu, (vm[0] & vm[1]) == 0xffffffffu);
      // 32-column chunks no row of this warp can see skip the max and the exponentials (P = 0)
      const unsigned vis_chunks = (__any_sync(0xffffffffu, vm[0] != 0u) ? 1u : 0u) |
                                  (__any_sync(0xffffffffu, vm[1] != 0u) ? 2u : 0u);
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
      if (warp_full) {
#pragma unroll
        for (int c = 0; c < 64; c += 2) mx[(c >> 1) & 7] = fmax3(mx[(c >> 1) & 7], s[c], s[c + 1]);
      } else {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          if (!((vis_chunks >> cc) & 1u)) continue;
#pragma unroll
          for (int x = 0; x < 32; x += 2) {
            const int c = cc * 32 + x;
            s[c] = (vm[cc] >> x) & 1u ? s[c] : -INFINITY;
            s[c + 1] = (vm[cc] >> (x + 1)) & 1u ? s[c + 1] : -INFINITY;
            mx[(x >> 1) & 7] = fmax3(mx[(x >> 1) & 7], s[c], s[c + 1]);
          }
        }
      }
      float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                         fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // the row max over both halves
      *red_at(it, hf) = mraw;
      tc::mbar_arrive(bar_x + q);
      ok = tc::mbar_wait(bar_x + q, it & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      mraw = fmaxf(mraw, *red_at(it, hf ^ 1));
      // raw-score max; the softmax scale (> 0) is folded into one FFMA before ex2
      const float m_cand = fmaxf(m_run, mraw * scale_log2);
      // lazy rescale: the running max moves only when the tile's max exceeds it by
      // more than 8 (log2 units), so P <= 2^8 and O is rescaled rarely
      const bool grow = m_cand > m_run + 8.f;
      const float m_new = grow ? m_cand : m_run;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float corr = grow ? ex2(m_run - m_use) : 1.f;
      // PV(it-1) of this query tile must be done before P(it) overwrites the P
      // buffer and O is rescaled (it was issued when P(it-1) was ready, so it is
      // normally complete by now; S(it+1) is already running on the tensor core)
      if (it > 0) {
        ok = tc::mbar_wait(bar_o_done + q, (it - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
      }
      uint64_t sm2[4] = {0ull, 0ull, 0ull, 0ull};  // packed partial row sums
      const uint64_t sc2 = f2(scale_log2, scale_log2), nm2 = f2(-m_use, -m_use);
      // P in 32-column pieces, each stored to shared memory (UMMA K-major) at once.
      // 6 of the 16 pairs of a piece are exponentiated on the FMA pipe, the
      // rest by MUFU, so neither unit alone sets the pace.
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t pk[16];
        if ((vis_chunks >> cc) & 1u) {
#pragma unroll
          for (int x = 0; x < 32; x += 2) {
            const int c = cc * 32 + x;
            float a, b, p0, p1;
            f2split(ffma2(f2(s[c], s[c + 1]), sc2, nm2), a, b);
            constexpr unsigned kPolyPairs = 0x2525u;  // pairs 0, 2, 5, 8, 10, 13 of 16
            if ((kPolyPairs >> (x >> 1)) & 1u) {
              exp2_poly2(a, b, p0, p1);
            } else {
              p0 = ex2(a);
              p1 = ex2(b);
            }
            sm2[(x >> 1) & 3] = fadd2(sm2[(x >> 1) & 3], f2(p0, p1));
            pk[x >> 1] = pack2(p0, p1);
          }
        } else {
#pragma unroll
          for (int x = 0; x < 16; ++x) pk[x] = 0u;
        }
        uint8_t* blk = sP + row * 128;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int ch = cc * 4 + q4;
          *reinterpret_cast<uint4*>(blk + ((ch ^ (row & 7)) << 4)) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        }
      }
      float sm[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) f2split(sm2[k], sm[2 * k], sm[2 * k + 1]);
      const float rs = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      l_run = l_run * corr + rs;  // this half's part of the row sum
      if (__any_sync(0xffffffffu, it > 0 && corr < 1.f)) {
        uint32_t r[32], r2[16];
        o_load(r, r2);
#pragma unroll
        for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * corr);
        tc::tmem_st32(tO, r);
        if constexpr (HO > 32) {
#pragma unroll
          for (int x = 0; x < 16; ++x) r2[x] = __float_as_uint(__uint_as_float(r2[x]) * corr);
          tc::tmem_st16(tO + 32, r2);
        }
        tc::tmem_wait_st();
      }
      m_run = m_new;
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_p_full + q);
    }
    if (ok && n_tiles > 0) {
      ok = tc::mbar_wait(bar_o_done + q, (n_tiles - 1) & 1, abort_flag, err);
      if (__all_sync(0xffffffffu, ok)) {
        // the row sum over both halves
        *red_at(n_tiles, hf) = l_run;
        tc::mbar_arrive(bar_x + q);
        ok = tc::mbar_wait(bar_x + q, n_tiles & 1, abort_flag, err);
        if (__all_sync(0xffffffffu, ok)) {
          const float l_tot = l_run + *red_at(n_tiles, hf ^ 1);
          tc::tc_fence_after();
          const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
          const int bq = bh / H, hq = bh % H;
          bf16* orow = O + (((int64_t)bq * Tn + i) * H + hq) * HD + hf * HO;
          uint32_t r[32], r2[16];
          o_load(r, r2);
          if (i < Tn) {
#pragma unroll
            for (int x = 0; x < 32; x += 8) {
              uint4 v = make_uint4(pack2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                                   pack2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                                   pack2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                                   pack2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
              *reinterpret_cast<uint4*>(orow + x) = v;
            }
            if constexpr (HO > 32) {
#pragma unroll
              for (int x = 0; x < 16; x += 8) {
                uint4 v = make_uint4(pack2(__uint_as_float(r2[x]) * inv, __uint_as_float(r2[x + 1]) * inv),
                                     pack2(__uint_as_float(r2[x + 2]) * inv, __uint_as_float(r2[x + 3]) * inv),
                                     pack2(__uint_as_float(r2[x + 4]) * inv, __uint_as_float(r2[x + 5]) * inv),
                                     pack2(__uint_as_float(r2[x + 6]) * inv, __uint_as_float(r2[x + 7]) * inv));
                *reinterpret_cast<uint4*>(orow + 32 + x) = v;
              }
            }
            if (hf == 0) LSE[(int64_t)bh * Tn + i] = (m_run + log2f(l_tot)) * 0.69314718055994531f;
          }
        }
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == MMA_WARP) tc::tmem_dealloc(tmem, TM_COLS);
}

// cuTensorMapEncodeTiled is a driver-API function; it is resolved at run time
// through the runtime's entry-point query so the library does not link libcuda
// (and still imports on a machine without a driver).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is not available from the CUDA driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// box_cols 64: 128-byte rows with the 128-byte swizzle; 32: 64-byte rows with the 64-byte swizzle
CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows,
                        uint32_t box_cols) {
  TORCH_CHECK(box_cols == 64 || box_cols == 32, "make_map_3d: box of 64 or 32 columns");
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, rows, outer};
  cuuint64_t strides[2] = {inner * 2, inner * rows * 2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows) {
  return make_map_3d(base, inner, rows, outer, box_rows, 64);
}

}  // namespace attn_tc

// device error word shared by the tcgen05 kernels (one per device)
at::Tensor& tc_error_word(const at::Device& dev) {
  static std::vector<at::Tensor> words(64);
  at::Tensor& w = words.at(dev.index());
  if (!w.defined()) w = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
  return w;
}

at::Tensor exp2_poly_eval(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat, "exp2_poly_eval: fp32 CUDA tensor");
  const at::cuda::CUDAGuard g(x.device());
  at::Tensor xc = x.contiguous();
  at::Tensor y = at::empty_like(xc);
  const int64_t n = xc.numel();
  if (n) attn_tc::exp2_poly_eval_kernel<<<(unsigned)((n / 2 + 255) / 256 + 1), 256, 0, stream()>>>(
             xc.data_ptr<float>(), y.data_ptr<float>(), n);
  check_launch("exp2_poly_eval");
  return y;
}

int64_t kernel_error_status(int64_t device, bool reset) {
  at::Tensor& w = tc_error_word(at::Device(at::kCUDA, (int)device));
  const int64_t v = w.item<int>();
  if (reset && v) w.zero_();
  return v;
}

bool attn_tc_supported(int64_t head_dim) { return head_dim == 64 || head_dim == 96; }  // backward
bool attn_tc_fwd_supported(int64_t head_dim) { return head_dim == 64 || head_dim == 96; }

// Same contract as attn_fwd_packed: Q [B,H,T,64], K/V [B,H,P+T,64] bf16 contiguous
// -> {O [B,T,H,64] bf16, LSE [B,H,T] fp32}
std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, int64_t window,
                                    double scale) {
  const at::cuda::CUDAGuard g(Q.device());
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && Q.is_contiguous() && K.is_contiguous() && V.is_contiguous(),
              "attn_fwd_tc: packed bf16 inputs");
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), hd = Q.size(3);
  TORCH_CHECK(hd == 64 || hd == 96, "attn_fwd_tc: head_dim must be 64 or 96");
  const int L = K.size(2), P = L - Tn;
  TORCH_CHECK(aligned16(Q) && aligned16(K) && aligned16(V), "attn_fwd_tc: 16-byte aligned inputs required");
  at::Tensor O = at::empty({B, Tn, H, hd}, Q.options());
  at::Tensor LSE = at::empty({B, H, Tn}, Q.options().dtype(at::kFloat));
  if ((int64_t)B * H * Tn == 0) return {O, LSE};
  const CUtensorMap mq = attn_tc::make_map_3d(Q.data_ptr(), hd, Tn, (uint64_t)B * H, attn_tc::BM);
  const CUtensorMap mk = attn_tc::make_map_3d(K.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN);
  const CUtensorMap mv = attn_tc::make_map_3d(V.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN);
  const int W = (int)std::min<int64_t>(window, 1 << 30);
  dim3 grid((Tn + attn_tc::NQ * attn_tc::BM - 1) / (attn_tc::NQ * attn_tc::BM), B * H);
  const float sl2 = (float)scale * 1.4426950408889634f;
  unsigned* err = (unsigned*)tc_error_word(Q.device()).data_ptr<int>();
  if (hd == 64) {
    static bool attr_set = false;
    if (!attr_set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_tc::attn_fwd_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          attn_tc::Fwd<64>::SMEM_BYTES));
      attr_set = true;
    }
    attn_tc::attn_fwd_tc_kernel<64><<<grid, attn_tc::NTHREADS, attn_tc::Fwd<64>::SMEM_BYTES, stream()>>>(
        mq, mk, mv, mq, mk, mv, (__nv_bfloat16*)O.data_ptr(), LSE.data_ptr<float>(), H, Tn, P, W, sl2, err);
  } else {
    // columns 64-95: 32-column boxes with the 64-byte swizzle, loaded at x = 64
    const CUtensorMap mq2 = attn_tc::make_map_3d(Q.data_ptr(), hd, Tn, (uint64_t)B * H, attn_tc::BM, 32);
    const CUtensorMap mk2 = attn_tc::make_map_3d(K.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN, 32);
    const CUtensorMap mv2 = attn_tc::make_map_3d(V.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN, 32);
    static bool attr_set = false;
    if (!attr_set) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(attn_tc::attn_fwd_tc_kernel<96>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          attn_tc::Fwd<96>::SMEM_BYTES));
      attr_set = true;
    }
    attn_tc::attn_fwd_tc_kernel<96><<<grid, attn_tc::NTHREADS, attn_tc::Fwd<96>::SMEM_BYTES, stream()>>>(
        mq, mk, mv, mq2, mk2, mv2, (__nv_bfloat16*)O.data_ptr(), LSE.data_ptr<float>(), H, Tn, P, W, sl2, err);
  }
  check_launch("attn_fwd_tc");
  return {O, LSE};
}

}  // namespace tb

namespace tb {

// =============================================================================
// Backward, head_dim 64, on tcgen05: a persistent kernel.
//
// Work item = one (batch, head), one tile of 128 keys (the M dimension of the
// key-major products) and a run of 128-query blocks that can see those keys
// (the tile holding the prefix keys, seen by every query, is split over
// several items).  The host builds the item list once per (T, P, window); each
// CTA (one per SM) walks items blockIdx.x, blockIdx.x + gridDim.x, ...
// 10 warps:
//   warp 8      TMA producer: K, V of each item into one of two slots (so the
//               next item's tiles land while this one finishes), and Q, dO,
//               log-sum-exp and D of each query block through a 2-stage ring;
//   warp 9      TMEM allocator + single-thread MMA issuer;
//   warps 0..7  two warpgroups of key-row threads: thread = key row = TMEM
//               lane; warpgroup w handles query columns [64w, 64w+64) of the
//               score tiles and column half w of the dQ / dK|dV drains.
// Per query block g (one global sequence over the CTA's items):
//   S^T  = K Q^T, dP^T = V dO^T     (M=128 keys, N=128 queries, K=64) -> TMEM
//   threads: P^T = exp2(S^T*scale*log2e - lse2), dS^T = P^T (dP^T - D) into
//            registers; release S^T/dP^T (s_free); store both as bf16 into
//            shared memory in the UMMA K-major layout (p_full); drain the
//            previous block's dQ rows (TMEM lane = query) with
//            red.global.add.v4.f32 into dQa (dq_free)
//   dV  += P^T dO, dK += dS^T Q     (M=128 keys, N=64, K=128; dO / Q MN-major)
//   dQ   = dS K                     (after dq_free; M=128 queries, N=64,
//                                    K=128 keys; dS read MN-major from the
//                                    dS^T tile)
// The MMA warp issues S/dP of block g+1 as soon as the threads have released
// block g's scores, so the tensor core computes the next scores while the
// threads store P/dS and drain dQ.  At the end of an item dK (scaled) and dV
// rows are stored (plain stores; vector reductions into rows zeroed by the
// pre-pass when the key tile is split over several items).
// All waits are bounded: a timeout records an error code and every role
// unwinds; TMEM is always released.
// =============================================================================
namespace attn_tcb {

using bf16 = __nv_bfloat16;
constexpr int HD = 64, BN = 128, BQ = 128;
constexpr int TILE = 128 * 64 * 2;  // 16 KB: one [128 rows][64 bf16] swizzled tile
constexpr int OFF_K = 0, OFF_V = OFF_K + 2 * TILE, OFF_Q = OFF_V + 2 * TILE, OFF_DO = OFF_Q + 2 * TILE;
constexpr int OFF_PT = OFF_DO + 2 * TILE, OFF_DST = OFF_PT + 2 * TILE;
constexpr int OFF_L = OFF_DST + 2 * TILE, OFF_D = OFF_L + 2 * BQ * 4, OFF_BAR = OFF_D + 2 * BQ * 4;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TM_ST = 0, TM_DPT = 128, TM_DV = 256, TM_DK = 320, TM_DQ = 384, TM_COLS = 512;
constexpr int QB_PER_SPLIT = 6;  // query blocks per item of a split key tile

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// 128-query blocks [qb_lo, qb_hi] that can see the key tile starting at
// combined key index n0 (P prefix keys, then the T sequence keys).
__host__ __device__ inline void tile_query_blocks(int n0, int P, int Tn, int W, int& qb_lo, int& qb_hi) {
  int q_lo, q_hi;
  if (n0 < P) {
    q_lo = 0;
    q_hi = Tn - 1;
  } else {
    const int last_key = (n0 + BN < P + Tn ? n0 + BN : P + Tn) - 1 - P;
    q_lo = n0 - P;
    q_hi = last_key + W - 1 < Tn - 1 ? last_key + W - 1 : Tn - 1;
  }
  qb_lo = q_lo / BQ;
  qb_hi = q_hi / BQ;
}

// D[bh, i] = sum_d dO * O and lse2 = LSE * log2(e) (both [BH][Tpad], zero
// padded); also zeroes the dQ accumulator and the dK/dV rows of split key
// tiles.  8 threads per row, RP rows per (batch, head).
__global__ void bwd_pre_tc_kernel(const bf16* __restrict__ dO, const bf16* __restrict__ O,
                                  const float* __restrict__ LSE, float* __restrict__ Dd, float* __restrict__ L2,
                                  float* __restrict__ dQa, float* __restrict__ dKa, float* __restrict__ dVa, int B,
                                  int H, int Tn, int Tpad, int P, int W, int RP) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r = e >> 3;
  const int c = (int)(e & 7);
  const int64_t bh = r / RP;
  const int i = (int)(r - bh * RP);
  const bool live = bh < (int64_t)B * H;
  float acc = 0.f;
  if (live && i < Tn) {
    const int b = (int)(bh / H), h = (int)(bh % H);
    const int64_t off = (((int64_t)b * Tn + i) * H + h) * HD + c * 8;
    float a[8], o[8];
    load16<bf16>(dO + off, a);
    load16<bf16>(O + off, o);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += a[k] * o[k];
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (!live) return;
  if (i < Tpad && c == 0) {
    Dd[bh * Tpad + i] = acc;
    L2[bh * Tpad + i] = i < Tn ? LSE[bh * Tn + i] * 1.4426950408889634f : 0.f;
  }
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i < Tn) {
    float4* q = reinterpret_cast<float4*>(dQa + (bh * Tn + i) * HD + c * 8);
    q[0] = z;
    q[1] = z;
  }
  if (i < P + Tn) {
    int lo, hi;
    tile_query_blocks(i / BN * BN, P, Tn, W, lo, hi);
    if (hi - lo + 1 > QB_PER_SPLIT) {
      const int64_t off = (bh * (P + Tn) + i) * HD + c * 8;
      reinterpret_cast<float4*>(dKa + off)[0] = z;
      reinterpret_cast<float4*>(dKa + off)[1] = z;
      reinterpret_cast<float4*>(dVa + off)[0] = z;
      reinterpret_cast<float4*>(dVa + off)[1] = z;
    }
  }
}

// Walks the query blocks of a CTA's items in order: item i = blockIdx.x,
// blockIdx.x + gridDim.x, ...; `it` counts the CTA's items, j the block within
// the item.  items[p] = {key tile, first query block, query blocks, split}.
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
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                       const int4* __restrict__ items, int n_pat, int n_items, const float* __restrict__ L2,
                       const float* __restrict__ Dd, float* __restrict__ dQa, float* __restrict__ dKa,
                       float* __restrict__ dVa, int H, int Tn, int Tpad, int P, int W, float scale,
                       float scale_log2, unsigned* __restrict__ err) {
  if ((int)blockIdx.x >= n_items) return;
  const int L = P + Tn;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* bar_kv_full = bars + 0;   // [2] K/V slot loaded
  uint64_t* bar_kv_empty = bars + 2;  // [2] K/V slot no longer read
  uint64_t* bar_q_full = bars + 4;    // [2]
  uint64_t* bar_q_empty = bars + 6;   // [2]
  uint64_t* bar_s_full = bars + 8;    // S^T, dP^T of the current block in TMEM
  uint64_t* bar_s_free = bars + 9;    // threads have read them
  uint64_t* bar_p_full = bars + 10;   // P^T, dS^T in shared memory; previous dQ drained
  uint64_t* bar_mma_done = bars + 11; // dV, dK, dQ of the block complete
  uint64_t* bar_dq_free = bars + 12;  // previous block's dQ drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(bar_kv_full + s, 1);
      tc::mbar_init(bar_kv_empty + s, 1);
      tc::mbar_init(bar_q_full + s, 1);
      tc::mbar_init(bar_q_empty + s, 1);
    }
    tc::mbar_init(bar_s_full, 1);
    tc::mbar_init(bar_s_free, 256);
    tc::mbar_init(bar_p_full, 256);
    tc::mbar_init(bar_mma_done, 1);
    tc::mbar_init(bar_dq_free, 256);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, TM_COLS);
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
      bool ok = true;
      while (ok && cur.valid()) {
        if (cur.j == 0) {
          const int slot = cur.it & 1;
          if (cur.it >= 2 && !tc::mbar_wait(bar_kv_empty + slot, ((cur.it >> 1) - 1) & 1, abort_flag, err)) break;
          tc::mbar_expect_tx(bar_kv_full + slot, 2 * TILE);
          tc::tma_load_3d(smem + OFF_K + slot * TILE, &tmK, bar_kv_full + slot, 0, cur.n0, cur.bh);
          tc::tma_load_3d(smem + OFF_V + slot * TILE, &tmV, bar_kv_full + slot, 0, cur.n0, cur.bh);
          ++kv_issued;
        }
        const int s = g & 1;
        if (g >= 2 && !tc::mbar_wait(bar_q_empty + s, ((g >> 1) - 1) & 1, abort_flag, err)) break;
        const int q0 = (cur.qs + cur.j) * BQ;
        const int b = cur.bh / H, h = cur.bh - b * H;
        tc::mbar_expect_tx(bar_q_full + s, 2 * TILE + 2 * BQ * 4);
        tc::tma_load_3d(smem + OFF_Q + s * TILE, &tmQ, bar_q_full + s, 0, q0, cur.bh);
        tc::tma_load_4d(smem + OFF_DO + s * TILE, &tmDO, bar_q_full + s, 0, h, q0, b);
        tc::bulk_load(smem + OFF_L + s * BQ * 4, L2 + (int64_t)cur.bh * Tpad + q0, BQ * 4, bar_q_full + s);
        tc::bulk_load(smem + OFF_D + s * BQ * 4, Dd + (int64_t)cur.bh * Tpad + q0, BQ * 4, bar_q_full + s);
        ++g;
        cur.next();
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA exits
        volatile int keep_waiting = 0;
        for (int t = max(0, kv_issued - 2); t < kv_issued; ++t)
          tc::mbar_wait(bar_kv_full + (t & 1), (t >> 1) & 1, &keep_waiting, nullptr, 1ll << 27);
        for (int t = max(0, g - 2); t < g; ++t)
          tc::mbar_wait(bar_q_full + (t & 1), (t >> 1) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t id_kv = tc::idesc_bf16_f32(128, HD, false, true);  // dV, dK: B (dO / Q) MN-major
      constexpr uint32_t id_q = tc::idesc_bf16_f32(128, HD, true, true);    // dQ: A (dS) and B (K) MN-major
      const uint32_t aK0 = tc::smem_addr(smem + OFF_K), aV0 = tc::smem_addr(smem + OFF_V);
      const uint32_t aPT = tc::smem_addr(smem + OFF_PT), aDST = tc::smem_addr(smem + OFF_DST);
      auto issue_sdp = [&](const Cursor& c, int gg) -> bool {
        const int s = gg & 1, slot = c.it & 1;
        if (c.j == 0 && !tc::mbar_wait(bar_kv_full + slot, (c.it >> 1) & 1, abort_flag, err)) return false;
        if (!tc::mbar_wait(bar_q_full + s, (gg >> 1) & 1, abort_flag, err)) return false;
        tc::tc_fence_after();
        const uint32_t aK = aK0 + slot * TILE, aV = aV0 + slot * TILE;
        const uint32_t aQ = tc::smem_addr(smem + OFF_Q + s * TILE), aDO = tc::smem_addr(smem + OFF_DO + s * TILE);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          tc::umma_bf16(tmem + TM_ST, tc::sdesc_sw128(aK + 32 * k, 16, 1024), tc::sdesc_sw128(aQ + 32 * k, 16, 1024),
                        id_s, k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          tc::umma_bf16(tmem + TM_DPT, tc::sdesc_sw128(aV + 32 * k, 16, 1024),
                        tc::sdesc_sw128(aDO + 32 * k, 16, 1024), id_s, k > 0);
        tc::umma_commit(bar_s_full);
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
        const int s = g & 1, slot = cur.it & 1;
        const uint32_t aK = aK0 + slot * TILE;
        const uint32_t aQ = tc::smem_addr(smem + OFF_Q + s * TILE), aDO = tc::smem_addr(smem + OFF_DO + s * TILE);
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          const uint32_t koff = (k >> 2) * (128 * 128) + (k & 3) * 32;  // K-major A: 64-query column blocks
          const uint32_t acc = (cur.j > 0 || k > 0) ? 1u : 0u;
          tc::umma_bf16(tmem + TM_DV, tc::sdesc_sw128(aPT + koff, 16, 1024),
                        tc::sdesc_sw128(aDO + k * 2048, 128 * 128, 1024), id_kv, acc);
          tc::umma_bf16(tmem + TM_DK, tc::sdesc_sw128(aDST + koff, 16, 1024),
                        tc::sdesc_sw128(aQ + k * 2048, 128 * 128, 1024), id_kv, acc);
        }
        if (!tc::mbar_wait(bar_dq_free, g & 1, abort_flag, err)) break;
        tc::tc_fence_after();
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          tc::umma_bf16(tmem + TM_DQ, tc::sdesc_sw128(aDST + k * 2048, 128 * 128, 1024),
                        tc::sdesc_sw128(aK + k * 2048, 128 * 128, 1024), id_q, k > 0);
        tc::umma_commit(bar_mma_done);
        tc::umma_commit(bar_q_empty + s);
        if (cur.j == cur.nq - 1) tc::umma_commit(bar_kv_empty + slot);
        cur = nxt;
      }
    }
  } else {
    // ------------------------------------------------------------ key-row threads
    const int wg = warp >> 2;
    const int r = threadIdx.x & 127;  // key row within the tile == TMEM lane
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    uint8_t* sPT = smem + OFF_PT;
    uint8_t* sDST = smem + OFF_DST;
    // dQ rows of query block q0 (TMEM lane = query row), column half wg
    auto drain_dq = [&](int bh, int q0) {
      const int i = q0 + r;
      uint32_t v[32];
      tc::tmem_ld32(tl + TM_DQ + wg * 32, v);
      tc::tmem_wait_ld();
      if (i < Tn) {
        float* dst = dQa + ((int64_t)bh * Tn + i) * HD + wg * 32;
#pragma unroll
        for (int x = 0; x < 32; x += 4)
          tc::red_add4(dst + x, __uint_as_float(v[x]) * scale, __uint_as_float(v[x + 1]) * scale,
                       __uint_as_float(v[x + 2]) * scale, __uint_as_float(v[x + 3]) * scale);
      }
    };
    Cursor cur(items, n_pat, n_items);
    for (int g = 0; cur.valid(); ++g) {
      const int s = g & 1;
      const int q0 = (cur.qs + cur.j) * BQ;
      const int jk = cur.n0 + r;  // combined key index of this thread's row
      bool ok = tc::mbar_wait(bar_s_full, g & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc::tc_fence_after();
      // visible query columns [c_lo, c_hi) of this key row in this block
      int c_lo = 0, c_hi = 0;
      if (jk < P) {
        c_hi = min(BQ, Tn - q0);
      } else if (jk < L) {
        const int jm = jk - P;
        c_lo = min(BQ, max(0, jm - q0));
        c_hi = max(c_lo, min(BQ, min(Tn - 1, jm + W - 1) - q0 + 1));
      }
      const float* sl = reinterpret_cast<const float*>(smem + OFF_L + s * BQ * 4);
      const float* sd = reinterpret_cast<const float*>(smem + OFF_D + s * BQ * 4);
      // every query column of the block visible to this key row: no masking
      const bool row_full = c_lo == 0 && c_hi == BQ;
      uint32_t pp[32], dd[32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = wg * 2 + cc;  // 32-query chunk handled by this warpgroup
        // no key row of this warp sees a query of the chunk (beyond the window, or
        // the non-prefix rows of the prefix tile): P^T = dS^T = 0 without the math
        if (!__any_sync(0xffffffffu, c_lo < c * 32 + 32 && c_hi > c * 32)) {
#pragma unroll
          for (int x = 0; x < 16; ++x) pp[cc * 16 + x] = dd[cc * 16 + x] = 0u;
          continue;
        }
        uint32_t st[32], dp[32];
        tc::tmem_ld32(tl + TM_ST + c * 32, st);
        tc::tmem_ld32(tl + TM_DPT + c * 32, dp);
        tc::tmem_wait_ld();
        const unsigned vm = row_full ? 0xffffffffu : attn_tc::range_bits(c_lo - c * 32, c_hi - c * 32);
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
      if (cur.j > 0) {
        // MMAs of the previous block done: P^T/dS^T buffers free, its dQ ready
        ok = tc::mbar_wait(bar_mma_done, (g - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc::tc_fence_after();
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = wg * 2 + cc;
        const int cb = c >> 1;  // 64-query column block
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (c & 1) * 4 + q;
          const int off = cb * (128 * 128) + r * 128 + ((ch ^ (r & 7)) << 4);
          const int u = cc * 16 + 4 * q;
          *reinterpret_cast<uint4*>(sPT + off) = make_uint4(pp[u], pp[u + 1], pp[u + 2], pp[u + 3]);
          *reinterpret_cast<uint4*>(sDST + off) = make_uint4(dd[u], dd[u + 1], dd[u + 2], dd[u + 3]);
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(bar_p_full);
      if (cur.j > 0) {
        drain_dq(cur.bh, q0 - BQ);
        tc::tc_fence_before();
      }
      tc::mbar_arrive(bar_dq_free);
      if (cur.j == cur.nq - 1) {
        // last block of the item: its dQ, then the item's dK (scaled,
        // warpgroup 0) and dV (warpgroup 1) rows
        ok = tc::mbar_wait(bar_mma_done, g & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) break;
        tc::tc_fence_after();
        drain_dq(cur.bh, q0);
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
  if (warp == 9) tc::tmem_dealloc(tmem, TM_COLS);
}

CUtensorMap make_map_dO(const void* base, int B, int Tn, int H) {
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)Tn, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)Tn * H * HD * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)BQ, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = attn_tc::encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dO) failed: ", (int)r);
  return m;
}

// Work items {key tile, first query block, query blocks, split} for one
// (T, P, window); the same list serves every (batch, head).  Cached per
// device and shape (built on the host once, then copied to the device).
const at::Tensor& work_items(const at::Device& dev, int Tn, int P, int W) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, at::Tensor> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_tuple((int)dev.index(), Tn, P, W);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  std::vector<int32_t> v;
  const int nkt = (P + Tn + BN - 1) / BN;
  for (int kt = 0; kt < nkt; ++kt) {
    int lo, hi;
    tile_query_blocks(kt * BN, P, Tn, W, lo, hi);
    const int nqb = hi - lo + 1;
    const int nsp = (nqb + QB_PER_SPLIT - 1) / QB_PER_SPLIT;
    const int per = (nqb + nsp - 1) / nsp;
    for (int sp = 0; sp < nsp; ++sp) {
      const int qs = lo + sp * per, qe = std::min(hi + 1, qs + per);
      if (qe <= qs) continue;
      v.insert(v.end(), {kt, qs, qe - qs, nsp > 1 ? 1 : 0});
    }
  }
  at::Tensor host = at::from_blob(v.data(), {(int64_t)v.size() / 4, 4}, at::kInt).clone();
  return cache.emplace(key, host.to(dev)).first->second;
}

}  // namespace attn_tcb

std::vector<at::Tensor> attn_bwd_tc96(const at::Tensor& dO_in, const at::Tensor& Q, const at::Tensor& K,
                                      const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE, int64_t window,
                                      double scale);

// Same contract as attn_bwd_packed (head_dim 64; head_dim 96 goes to
// attn_bwd_tc96): returns {dQa, dKa, dVa} fp32.
std::vector<at::Tensor> attn_bwd_tc(const at::Tensor& dO_in, const at::Tensor& Q, const at::Tensor& K,
                                    const at::Tensor& V, const at::Tensor& O, const at::Tensor& LSE, int64_t window,
                                    double scale) {
  using namespace attn_tcb;
  if (Q.size(3) == 96) return attn_bwd_tc96(dO_in, Q, K, V, O, LSE, window, scale);
  const at::cuda::CUDAGuard g(Q.device());
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), hd = Q.size(3);
  TORCH_CHECK(hd == HD, "attn_bwd_tc: head_dim must be 64");
  const int L = K.size(2), P = L - Tn;
  at::Tensor dO = dO_in.to(at::kBFloat16).contiguous();
  TORCH_CHECK(dO.sizes() == O.sizes() && aligned16(dO) && aligned16(Q) && aligned16(K) && aligned16(V),
              "attn_bwd_tc: layout");
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
    const int64_t work = (int64_t)B * H * RP * 8;
    bwd_pre_tc_kernel<<<(work + 255) / 256, 256, 0, stream()>>>(
        (const bf16*)dO.data_ptr(), (const bf16*)O.data_ptr(), LSE.data_ptr<float>(), Dd.data_ptr<float>(),
        L2.data_ptr<float>(), dQa.data_ptr<float>(), dKa.data_ptr<float>(), dVa.data_ptr<float>(), B, H, Tn, Tpad,
        P, W, RP);
    check_launch("attn_bwd_tc pre");
  }
  const at::Tensor& items = work_items(Q.device(), Tn, P, W);
  const int n_pat = items.size(0);
  const int64_t n_items64 = (int64_t)n_pat * B * H;
  TORCH_CHECK(n_items64 < (1ll << 31), "attn_bwd_tc: too many work items");
  const int n_items = (int)n_items64;
  const CUtensorMap mk = attn_tc::make_map_3d(K.data_ptr(), HD, L, (uint64_t)B * H, BN);
  const CUtensorMap mv = attn_tc::make_map_3d(V.data_ptr(), HD, L, (uint64_t)B * H, BN);
  const CUtensorMap mq = attn_tc::make_map_3d(Q.data_ptr(), HD, Tn, (uint64_t)B * H, BQ);
  const CUtensorMap mdo = make_map_dO(dO.data_ptr(), B, Tn, H);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set = true;
  }
  const int grid = std::min(n_items, num_sms());
  attn_bwd_tc_kernel<<<grid, 320, SMEM_BYTES, stream()>>>(
      mk, mv, mq, mdo, reinterpret_cast<const int4*>(items.data_ptr<int>()), n_pat, n_items, L2.data_ptr<float>(),
      Dd.data_ptr<float>(), dQa.data_ptr<float>(), dKa.data_ptr<float>(), dVa.data_ptr<float>(), H, Tn, Tpad, P, W,
      (float)scale, (float)scale * 1.4426950408889634f, (unsigned*)tc_error_word(Q.device()).data_ptr<int>());
  check_launch("attn_bwd_tc");
  return {dQa, dKa, dVa};
}

}  // namespace tb
