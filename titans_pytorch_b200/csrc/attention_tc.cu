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
#include "tc_common.cuh"

namespace tb {
namespace attn_tc {

using bf16 = __nv_bfloat16;

constexpr int HD = 64;
constexpr int BM = 128;  // rows per query tile
constexpr int NQ = 2;    // query tiles per CTA
constexpr int BN = 128;  // keys per tile
constexpr int NS = 2;    // K/V stages
constexpr int TILE_Q = BM * HD * 2;
constexpr int TILE_K = BN * HD * 2;
constexpr int TILE_P = BM * BN * 2;
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NQ * TILE_Q;
constexpr int OFF_V = OFF_K + NS * TILE_K;
constexpr int OFF_P = OFF_V + NS * TILE_K;
constexpr int OFF_BAR = OFF_P + NQ * TILE_P;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TM_S = 0, TM_O = 256, TM_COLS = 512;
constexpr int NTHREADS = 320;

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(NTHREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, bf16* __restrict__ O, float* __restrict__ LSE,
                       int H, int Tn, int P, int W, float scale_log2, unsigned* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* bar_q = bars + 0;
  uint64_t* bar_kv_full = bars + 1;          // [NS]
  uint64_t* bar_kv_empty = bars + 1 + NS;    // [NS]
  uint64_t* bar_s_full = bars + 1 + 2 * NS;  // [NQ]
  uint64_t* bar_p_full = bars + 3 + 2 * NS;  // [NQ]
  uint64_t* bar_o_done = bars + 5 + 2 * NS;  // [NQ]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
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
      tc::mbar_init(bar_p_full + q, 128);
      tc::mbar_init(bar_o_done + q, 1);
    }
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
    if (lane == 0 && n_tiles > 0) {
      tc::tma_prefetch_desc(&tmQ);
      tc::tma_prefetch_desc(&tmK);
      tc::tma_prefetch_desc(&tmV);
      tc::mbar_expect_tx(bar_q, NQ * TILE_Q);
      for (int q = 0; q < NQ; ++q) tc::tma_load_3d(smem + OFF_Q + q * TILE_Q, &tmQ, bar_q, 0, m0 + q * BM, bh);
      int issued = 0;
      for (int it = 0; it < n_tiles; ++it) {
        const int s = it % NS;
        if (it >= NS && !tc::mbar_wait(bar_kv_empty + s, ((it / NS) - 1) & 1, abort_flag, err)) break;
        const int n0 = tile_n0(it);
        tc::mbar_expect_tx(bar_kv_full + s, 2 * TILE_K);
        tc::tma_load_3d(smem + OFF_K + s * TILE_K, &tmK, bar_kv_full + s, 0, n0, bh);
        tc::tma_load_3d(smem + OFF_V + s * TILE_K, &tmV, bar_kv_full + s, 0, n0, bh);
        issued = it + 1;
      }
      if (*abort_flag) {
        volatile int keep_waiting = 0;  // let issued copies land before exit (bounded)
        for (int it = max(0, issued - NS); it < issued; ++it)
          tc::mbar_wait(bar_kv_full + (it % NS), (it / NS) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_o = tc::idesc_bf16_f32(BM, HD, false, true);
      bool ok = tc::mbar_wait(bar_q, 0, abort_flag, err);
      auto issue_s = [&](int q, int it) {
        const uint32_t aQ = tc::smem_addr(smem + OFF_Q + q * TILE_Q);
        const uint32_t aK = tc::smem_addr(smem + OFF_K + (it % NS) * TILE_K);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          tc::umma_bf16(tmem + TM_S + q * BN, tc::sdesc_sw128(aQ + 32 * k, 16, 1024),
                        tc::sdesc_sw128(aK + 32 * k, 16, 1024), idesc_s, k > 0);
        tc::umma_commit(bar_s_full + q);
      };
      if (ok) ok = tc::mbar_wait(bar_kv_full, 0, abort_flag, err);
      if (ok) {
        tc::tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int it = 0; ok && it < n_tiles; ++it) {
        const int s = it % NS;
        const bool more = it + 1 < n_tiles;
        const uint32_t aV = tc::smem_addr(smem + OFF_V + s * TILE_K);
        for (int q = 0; q < NQ && ok; ++q) {
          if (!tc::mbar_wait(bar_p_full + q, it & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t aP = tc::smem_addr(smem + OFF_P + q * TILE_P);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint64_t ad = tc::sdesc_sw128(aP + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = tc::sdesc_sw128(aV + k * 2048, BN * 128, 1024);  // V: MN-major
            tc::umma_bf16(tmem + TM_O + q * HD, ad, bd, idesc_o, (it > 0 || k > 0) ? 1u : 0u);
          }
          tc::umma_commit(bar_o_done + q);
          if (q == NQ - 1) tc::umma_commit(bar_kv_empty + s);
          if (more) {
            if (q == 0) {
              if (!tc::mbar_wait(bar_kv_full + ((it + 1) % NS), ((it + 1) / NS) & 1, abort_flag, err)) {
                ok = false;
                break;
              }
              tc::tc_fence_after();
            }
            issue_s(q, it + 1);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int q = warp >> 2;              // query tile of this warpgroup
    const int row = threadIdx.x & 127;    // TMEM lane
    const int i = m0 + q * BM + row;      // query index
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t tS = tl + TM_S + q * BN, tO = tl + TM_O + q * HD;
    uint8_t* sP = smem + OFF_P + q * TILE_P;
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
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(tS + c * 32, r);
#pragma unroll
        for (int x = 0; x < 32; ++x) s[c * 32 + x] = __uint_as_float(r[x]);
      }
      tc::tmem_wait_ld();
      // visible columns: [0, pre_hi) are prefix keys; [lo2, hi2) the window
      const int pre_hi = min(BN, max(0, P - n0));
      const int lo2 = max(pre_hi, P - n0 + win_lo);
      const int hi2 = min(BN, P - n0 + win_hi + 1);
      const bool row_full = (pre_hi >= BN) || (lo2 <= pre_hi && pre_hi == 0 && lo2 <= 0 && hi2 >= BN);
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
      if (__all_sync(0xffffffffu, row_full)) {
        // every row of this warp sees the whole tile: no masking
#pragma unroll
        for (int c = 0; c < BN; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
      } else {
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const bool vis = (c < pre_hi) | ((c >= lo2) & (c < hi2));
          s[c] = vis ? s[c] : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], s[c]);
        }
      }
      // raw-score max; the softmax scale (> 0) is folded into one FFMA before ex2
      const float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const float m_new = fmaxf(m_run, mraw * scale_log2);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float corr = ex2(m_run - m_use);
      float sm[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) sm[k] = 0.f;
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = ex2(fmaf(s[c], scale_log2, -m_use)), p1 = ex2(fmaf(s[c + 1], scale_log2, -m_use));
        sm[(c >> 1) & 7] += p0 + p1;
        pk[c / 2] = pack2(p0, p1);
      }
      const float rs = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      l_run = l_run * corr + rs;
      // PV(it-1) of this tile done: O is stable and the P buffer is free
      if (it > 0) {
        ok = tc::mbar_wait(bar_o_done + q, (it - 1) & 1, abort_flag, err);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
      }
#pragma unroll
      for (int cb = 0; cb < 2; ++cb)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int x = cb * 32 + ch * 4;
          *reinterpret_cast<uint4*>(sP + cb * (BM * 128) + row * 128 + ((ch ^ (row & 7)) << 4)) =
              make_uint4(pk[x], pk[x + 1], pk[x + 2], pk[x + 3]);
        }
      if (__any_sync(0xffffffffu, it > 0 && corr < 1.f)) {
#pragma unroll
        for (int h = 0; h < HD / 32; ++h) {
          uint32_t r[32];
          tc::tmem_ld32(tO + h * 32, r);
          tc::tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * corr);
          tc::tmem_st32(tO + h * 32, r);
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
        tc::tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        const int bq = bh / H, hq = bh % H;
        bf16* orow = O + (((int64_t)bq * Tn + i) * H + hq) * HD;
#pragma unroll
        for (int h = 0; h < HD / 32; ++h) {
          uint32_t r[32];
          tc::tmem_ld32(tO + h * 32, r);
          tc::tmem_wait_ld();
          if (i < Tn) {
#pragma unroll
            for (int x = 0; x < 32; x += 8) {
              uint4 v = make_uint4(pack2(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv),
                                   pack2(__uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv),
                                   pack2(__uint_as_float(r[x + 4]) * inv, __uint_as_float(r[x + 5]) * inv),
                                   pack2(__uint_as_float(r[x + 6]) * inv, __uint_as_float(r[x + 7]) * inv));
              *reinterpret_cast<uint4*>(orow + h * 32 + x) = v;
            }
          }
        }
        if (i < Tn) LSE[(int64_t)bh * Tn + i] = (m_run + log2f(l_run)) * 0.69314718055994531f;
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 9) tc::tmem_dealloc(tmem, TM_COLS);
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

CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, rows, outer};
  cuuint64_t strides[2] = {inner * 2, inner * rows * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

}  // namespace attn_tc

// device error word shared by the tcgen05 kernels (one per device)
at::Tensor& tc_error_word(const at::Device& dev) {
  static std::vector<at::Tensor> words(64);
  at::Tensor& w = words.at(dev.index());
  if (!w.defined()) w = at::zeros({1}, at::TensorOptions().device(dev).dtype(at::kInt));
  return w;
}

int64_t kernel_error_status(int64_t device, bool reset) {
  at::Tensor& w = tc_error_word(at::Device(at::kCUDA, (int)device));
  const int64_t v = w.item<int>();
  if (reset && v) w.zero_();
  return v;
}

bool attn_tc_supported(int64_t head_dim) { return head_dim == attn_tc::HD; }

// Same contract as attn_fwd_packed: Q [B,H,T,64], K/V [B,H,P+T,64] bf16 contiguous
// -> {O [B,T,H,64] bf16, LSE [B,H,T] fp32}
std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, int64_t window,
                                    double scale) {
  const at::cuda::CUDAGuard g(Q.device());
  TORCH_CHECK(Q.scalar_type() == at::kBFloat16 && Q.is_contiguous() && K.is_contiguous() && V.is_contiguous(),
              "attn_fwd_tc: packed bf16 inputs");
  const int B = Q.size(0), H = Q.size(1), Tn = Q.size(2), hd = Q.size(3);
  TORCH_CHECK(hd == attn_tc::HD, "attn_fwd_tc: head_dim must be 64");
  const int L = K.size(2), P = L - Tn;
  TORCH_CHECK(aligned16(Q) && aligned16(K) && aligned16(V), "attn_fwd_tc: 16-byte aligned inputs required");
  at::Tensor O = at::empty({B, Tn, H, hd}, Q.options());
  at::Tensor LSE = at::empty({B, H, Tn}, Q.options().dtype(at::kFloat));
  if ((int64_t)B * H * Tn == 0) return {O, LSE};
  const CUtensorMap mq = attn_tc::make_map_3d(Q.data_ptr(), hd, Tn, (uint64_t)B * H, attn_tc::BM);
  const CUtensorMap mk = attn_tc::make_map_3d(K.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN);
  const CUtensorMap mv = attn_tc::make_map_3d(V.data_ptr(), hd, L, (uint64_t)B * H, attn_tc::BN);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(attn_tc::attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         attn_tc::SMEM_BYTES);
    attr_set = true;
  }
  const int W = (int)std::min<int64_t>(window, 1 << 30);
  dim3 grid((Tn + attn_tc::NQ * attn_tc::BM - 1) / (attn_tc::NQ * attn_tc::BM), B * H);
  attn_tc::attn_fwd_tc_kernel<<<grid, attn_tc::NTHREADS, attn_tc::SMEM_BYTES, stream()>>>(
      mq, mk, mv, (__nv_bfloat16*)O.data_ptr(), LSE.data_ptr<float>(), H, Tn, P, W,
      (float)scale * 1.4426950408889634f, (unsigned*)tc_error_word(Q.device()).data_ptr<int>());
  check_launch("attn_fwd_tc");
  return {O, LSE};
}

}  // namespace tb
