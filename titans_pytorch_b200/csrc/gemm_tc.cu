// Persistent tcgen05 GEMM, C[M, N] (bf16) = A[M, K] . B[N, K]^T (both bf16,
// K contiguous, fp32 accumulation in TMEM), optionally fused with the
// all-gather of a sharded parameter unit that contains B.
//
// Layout of one CTA (one per SM, persistent over output tiles of 128 x 256):
//   warp 0      TMA producer: A and B k-slices (64 columns, 128-byte swizzle)
//               into a 4-stage shared-memory ring
//   warp 1      TMEM allocator and MMA issuer (one thread): 4 x tcgen05.mma
//               (M=128, N=256, K=16) per k-slice into one of two TMEM
//               accumulators (2 x 256 columns), so the epilogue of a tile
//               overlaps the next tile's MMAs
//   warps 2-5   epilogue: thread = accumulator row (TMEM lane), tcgen05.ld of
//               32 columns at a time, bf16 conversion, 64-byte row stores
//               (8 warps splitting the columns measured slower)
//   warp 6      gather (fused mode only)
//
// Fused all-gather.  The parameters of a unit (flat elements [u0, u0 + len)
// of a flat buffer laid out identically on every rank) are sharded: rank r
// holds the current values of unit elements [r * shard, (r + 1) * shard).
// The gather warp of CTA c copies the 16 KB pieces q = c, c + grid, ... of
// the unit from their owners' buffers (peer pointers, plain
// cp.async.bulk global -> shared, no multicast) and writes them into this
// rank's buffer (cp.async.bulk shared -> global), so each remote byte crosses
// NVLink once and the tensor-core tiles run meanwhile.  Two uses:
//   * consume: B lies inside the unit.  Pieces are visited starting at the
//     one holding B, so B's rows land first; after a piece is written the
//     counter of every 256-row block of B it overlaps is incremented
//     (release), and the producer waits (acquire, bounded) until its row
//     block's counter equals the number of pieces covering it before loading
//     B from local memory by TMA.  Launched cooperatively (all CTAs
//     resident), so a CTA waiting for another CTA's piece cannot starve it.
//   * prefetch: B is already local (the current layer's weights) and the
//     unit is the next layer's; nothing waits.
//
// All waits are bounded: a timeout records an error code in the error word and
// the CTA unwinds (bounded wait for its in-flight copies, TMEM freed).
#include "tc_common.cuh"

namespace tb {

namespace attn_tc {
CUtensorMap make_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t outer, uint32_t box_rows);
}
at::Tensor& tc_error_word(const at::Device& dev);

namespace gemm_k {

constexpr int BM = 128, BN = 256, BK = 64, NS = 4;
constexpr int TILE_A = BM * BK * 2, TILE_B = BN * BK * 2, STAGE = TILE_A + TILE_B;
constexpr int PIECE = 8192;  // gather piece, elements (16 KB)
constexpr int PIECE_BYTES = PIECE * 2;
constexpr int OFF_G = NS * STAGE;
constexpr int OFF_BAR = OFF_G + 2 * PIECE_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // barriers + alignment slack
constexpr int EPI_WARPS = 4;  // a multiple of 4 (one warp per TMEM lane quarter and column slice)
constexpr int EPI_CHUNKS = BN / 32 / (EPI_WARPS / 4);  // 32-column chunks per epilogue warp
constexpr int NTHREADS = 32 * (3 + EPI_WARPS);
constexpr int TM_COLS = 2 * BN;

enum : unsigned { ERR_GATHER_WAIT = 40 };

struct Gather {
  const __nv_bfloat16* const* src;  // [world] every rank's flat buffer (peer pointers; own entry local)
  __nv_bfloat16* dst;               // this rank's flat buffer; nullptr: no gather
  unsigned* counts;                 // consume mode: [ceil(N / BN)] pieces landed per B row block (zeroed
                                    // before launch); nullptr: B is not waited for
  int64_t u0, len, shard, w0;       // unit [u0, u0 + len); rank r owns [r * shard, (r + 1) * shard); B at w0
  int world, me;
  int copy_own;                     // also copy this rank's own part (the unit's destination is a working
                                    // slot, its source this rank's shard store)
};

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(tc::smem_addr(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

// pieces (unit-relative index) covering B's row block nt
__device__ __forceinline__ unsigned pieces_of_block(const Gather& g, int nt, int N, int K) {
  const int64_t wl = g.w0 - g.u0;
  const int64_t lo = wl + (int64_t)nt * BN * K, hi = wl + (int64_t)min(N, (nt + 1) * BN) * K;
  return (unsigned)((hi - 1) / PIECE - lo / PIECE + 1);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   __nv_bfloat16* __restrict__ C, int M, int N, int K, const Gather g, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* bar_empty = bar_full + NS;
  uint64_t* bar_acc_full = bar_empty + NS;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_g = bar_acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_g + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mt = (M + BM - 1) / BM, n_nt = (N + BN - 1) / BN, tiles = n_mt * n_nt;
  const int nk = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + s, 1);
      tc::mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_acc_full + b, 1);
      tc::mbar_init(bar_acc_empty + b, 32 * EPI_WARPS);
      tc::mbar_init(bar_g + b, 1);
    }
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, TM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmA);
      tc::tma_prefetch_desc(&tmB);
      uint64_t seen = 0;  // row blocks of B already known to be gathered (n_nt <= 64 tracked)
      int it = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mt = t / n_nt, nt = t % n_nt;
        if (g.counts != nullptr && !(nt < 64 && ((seen >> nt) & 1ull))) {
          const unsigned want = pieces_of_block(g, nt, N, K);
          const long long t0 = clock64();
          while (ld_acquire_gpu(g.counts + nt) < want) {
            if (*abort_flag) { ok = false; break; }
            if (clock64() - t0 > (1ll << 31)) {
              *abort_flag = 1;
              tc::set_error(err, ERR_GATHER_WAIT);
              ok = false;
              break;
            }
          }
          if (!ok) break;
          fence_proxy_async_global();  // generic-proxy writes of the gather before async-proxy TMA reads
          if (nt < 64) seen |= 1ull << nt;
        }
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % NS;
          if (it >= NS && !tc::mbar_wait(bar_empty + s, ((it / NS) - 1) & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          tc::mbar_expect_tx(bar_full + s, STAGE);
          tc::tma_load_3d(smem + s * STAGE, &tmA, bar_full + s, kc * BK, mt * BM, 0);
          tc::tma_load_3d(smem + s * STAGE + TILE_A, &tmB, bar_full + s, kc * BK, nt * BN, 0);
          issued = it + 1;
        }
      }
      if (*abort_flag) {
        volatile int keep_waiting = 0;  // let issued copies land before exit (bounded)
        for (int i = max(0, issued - NS); i < issued; ++i)
          tc::mbar_wait(bar_full + (i % NS), (i / NS) & 1, &keep_waiting, nullptr, 1ll << 27);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, false, false);
      int it = 0, li = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++li) {
        const int buf = li & 1;
        if (li >= 2 && !tc::mbar_wait(bar_acc_empty + buf, ((li >> 1) - 1) & 1, abort_flag, err)) break;
        tc::tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % NS;
          if (!tc::mbar_wait(bar_full + s, (it / NS) & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t aA = tc::smem_addr(smem + s * STAGE), aB = aA + TILE_A;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc::umma_bf16(d, tc::sdesc_sw128(aA + 32 * k, 16, 1024), tc::sdesc_sw128(aB + 32 * k, 16, 1024), idesc,
                          (kc > 0 || k > 0) ? 1u : 0u);
          tc::umma_commit(bar_empty + s);
        }
        if (ok) tc::umma_commit(bar_acc_full + buf);
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int slice = (warp - 2) >> 2;  // column slice of the tile
    const int r_in = q * 32 + lane;
    int li = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++li) {
      const int buf = li & 1;
      if (!tc::mbar_wait(bar_acc_full + buf, (li >> 1) & 1, abort_flag, err)) break;
      tc::tc_fence_after();
      const int mt = t / n_nt, nt = t % n_nt;
      const int row = mt * BM + r_in;
      __nv_bfloat16* crow = C + (int64_t)row * N + nt * BN;
#pragma unroll 1
      for (int c = slice * EPI_CHUNKS; c < (slice + 1) * EPI_CHUNKS; ++c) {
        const int col0 = nt * BN + c * 32;
        if (col0 >= N) break;  // warp-uniform
        uint32_t r[32];
        tc::tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * BN + c * 32, r);
        tc::tmem_wait_ld();
        if (row < M) {
          uint32_t p[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) p[j] = pack_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          uint4* dst = reinterpret_cast<uint4*>(crow + c * 32);
          if (col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
          } else {
            for (int j = 0; j < 4 && col0 + 8 * j < N; ++j)
              dst[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(bar_acc_empty + buf);
    }
  } else if (g.dst != nullptr && lane == 0) {
    // ------------------------------------------------------------ gather (warp 6)
    const int64_t n_pieces = (g.len + PIECE - 1) / PIECE;
    const int64_t p_first = g.counts != nullptr ? (g.w0 - g.u0) / PIECE : 0;
    const int64_t wl = g.w0 - g.u0, wh = wl + (int64_t)N * K, rb = (int64_t)BN * K;
    auto piece_of = [&](int64_t q) { return (p_first + q) % n_pieces; };
    // remote segments of piece p: [e, e_end) owned by r != me
    auto issue = [&](int64_t q, int b) -> uint32_t {
      const int64_t p = piece_of(q);
      const int64_t e0 = p * PIECE, e1 = min(e0 + PIECE, g.len);
      uint32_t bytes = 0;
      for (int64_t e = e0; e < e1;) {
        const int owner = (int)(e / g.shard);
        const int64_t se = min(e1, (int64_t)(owner + 1) * g.shard);
        if (owner != g.me || g.copy_own) bytes += (uint32_t)((se - e) * 2);
        e = se;
      }
      if (bytes == 0) return 0;
      tc::mbar_expect_tx(bar_g + b, bytes);
      for (int64_t e = e0; e < e1;) {
        const int owner = (int)(e / g.shard);
        const int64_t se = min(e1, (int64_t)(owner + 1) * g.shard);
        if (owner != g.me || g.copy_own)
          tc::bulk_load(smem + OFF_G + b * PIECE_BYTES + (e - e0) * 2, g.src[owner] + g.u0 + e, (uint32_t)((se - e) * 2),
                        bar_g + b);
        e = se;
      }
      return bytes;
    };
    uint32_t pend[2] = {0, 0};
    int uses[2] = {0, 0};
    int64_t q = blockIdx.x;
    if (q < n_pieces) pend[0] = issue(q, 0);
    bool ok = true;
    for (int j = 0; q < n_pieces; ++j, q += gridDim.x) {
      const int b = j & 1;
      const int64_t qn = q + gridDim.x;
      pend[b ^ 1] = (ok && qn < n_pieces) ? issue(qn, b ^ 1) : 0u;
      const int64_t p = piece_of(q);
      const int64_t e0 = p * PIECE, e1 = min(e0 + PIECE, g.len);
      if (pend[b]) {
        ok = ok && tc::mbar_wait(bar_g + b, uses[b] & 1, abort_flag, err);
        if (!ok) {  // the load is still in flight: let it land (bounded) before the CTA exits
          volatile int keep_waiting = 0;
          tc::mbar_wait(bar_g + b, uses[b] & 1, &keep_waiting, nullptr, 1ll << 27);
        }
        ++uses[b];
        pend[b] = 0;
        if (ok) {
          for (int64_t e = e0; e < e1;) {
            const int owner = (int)(e / g.shard);
            const int64_t se = min(e1, (int64_t)(owner + 1) * g.shard);
            if (owner != g.me || g.copy_own) bulk_store(g.dst + g.u0 + e, smem + OFF_G + b * PIECE_BYTES + (e - e0) * 2,
                                          (uint32_t)((se - e) * 2));
            e = se;
          }
          bulk_commit();
          bulk_wait_all();
          fence_proxy_async_global();
        }
      }
      if (!ok) {
        if (pend[b ^ 1]) {
          volatile int keep_waiting = 0;
          tc::mbar_wait(bar_g + (b ^ 1), uses[b ^ 1] & 1, &keep_waiting, nullptr, 1ll << 27);
        }
        break;
      }
      const int64_t lo = max(e0, wl), hi = min(e1, wh);
      if (g.counts != nullptr && lo < hi) {
        const int nt0 = (int)((lo - wl) / rb), nt1 = (int)((hi - 1 - wl) / rb);
        __threadfence();
        for (int nt = nt0; nt <= nt1; ++nt) red_release_gpu_add(g.counts + nt, 1u);
      }
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace gemm_k

namespace {

void launch_gemm(const at::Tensor& A, const __nv_bfloat16* Bptr, at::Tensor& Cout, int M, int N, int K,
                 const gemm_k::Gather& g, const at::Device& dev) {
  using namespace gemm_k;
  const CUtensorMap ma = attn_tc::make_map_3d(A.data_ptr(), K, M, 1, BM);
  const CUtensorMap mb = attn_tc::make_map_3d(Bptr, K, N, 1, BN);
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = g.dst != nullptr ? num_sms() : std::min(tiles, num_sms());
  unsigned* err = (unsigned*)tc_error_word(dev).data_ptr<int>();
  __nv_bfloat16* C = (__nv_bfloat16*)Cout.data_ptr();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = g.counts != nullptr ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tc_kernel, ma, mb, C, M, N, K, g, err));
}

void check_operand(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "gemm_tc: ", what,
              " must be a contiguous bf16 CUDA tensor");
  TORCH_CHECK(aligned16(t), "gemm_tc: ", what, " must be 16-byte aligned");
}

}  // namespace

// C = A . B^T, A [M, K], B [N, K] (bf16, K a multiple of 8, N a multiple of 8)
at::Tensor gemm_tc(const at::Tensor& A, const at::Tensor& B) {
  const at::cuda::CUDAGuard guard(A.device());
  check_operand(A, "A");
  check_operand(B, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_tc: A [M, K], B [N, K]");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "gemm_tc: K and N must be multiples of 8");
  at::Tensor Cout = at::empty({M, N}, A.options());
  if (M == 0 || N == 0) return Cout;
  if (K == 0) return Cout.zero_();
  gemm_k::Gather g{};
  launch_gemm(A, (const __nv_bfloat16*)B.data_ptr(), Cout, M, N, K, g, A.device());
  check_launch("gemm_tc");
  return Cout;
}

// Fused all-gather + GEMM: C = A . B^T while unit [u0, u0 + len) of this
// rank's flat bf16 buffer `flat` is gathered from every rank's buffer
// (`src_ptrs`, int64 [world] on the device; rank r owns unit-relative
// [r * shard, (r + 1) * shard)).  `consume`: B is a view of `flat` inside the
// unit and its tiles wait for their rows; otherwise B is any local tensor
// (prefetch of another layer's parameters).
at::Tensor gemm_gather_tc(const at::Tensor& A, const at::Tensor& B, at::Tensor& flat, const at::Tensor& src_ptrs,
                          int64_t u0, int64_t len, int64_t shard, int64_t me, bool consume, bool copy_own) {
  const at::cuda::CUDAGuard guard(A.device());
  check_operand(A, "A");
  check_operand(B, "B");
  TORCH_CHECK(flat.is_cuda() && flat.scalar_type() == at::kBFloat16 && flat.is_contiguous() && aligned16(flat),
              "gemm_gather_tc: flat must be a contiguous bf16 CUDA buffer");
  TORCH_CHECK(src_ptrs.is_cuda() && src_ptrs.scalar_type() == at::kLong, "gemm_gather_tc: src_ptrs int64 on device");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_gather_tc: A [M, K], B [N, K]");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(M > 0 && K % 8 == 0 && N % 8 == 0, "gemm_gather_tc: M > 0, K and N multiples of 8");
  TORCH_CHECK(u0 % 8 == 0 && len % 8 == 0 && shard % 8 == 0 && shard > 0 && len > 0 && u0 + len <= flat.numel(),
              "gemm_gather_tc: unit must be 8-element aligned and inside the buffer");
  const int world = (int)src_ptrs.numel();
  TORCH_CHECK(shard * world >= len && me >= 0 && me < world, "gemm_gather_tc: shard layout");
  const auto* fb = (const __nv_bfloat16*)flat.data_ptr();
  const auto* bp = (const __nv_bfloat16*)B.data_ptr();
  const int64_t w0 = bp - fb;
  if (consume)
    TORCH_CHECK(bp >= fb && w0 >= u0 && w0 + N * K <= u0 + len && w0 % 8 == 0,
                "gemm_gather_tc: consume mode needs B inside the gathered unit");
  at::Tensor Cout = at::empty({M, N}, A.options());
  at::Tensor counts;
  if (consume) counts = at::zeros({(N + gemm_k::BN - 1) / gemm_k::BN}, A.options().dtype(at::kInt));
  gemm_k::Gather g;
  g.src = reinterpret_cast<const __nv_bfloat16* const*>(src_ptrs.data_ptr<int64_t>());
  g.dst = (__nv_bfloat16*)flat.data_ptr();
  g.counts = consume ? (unsigned*)counts.data_ptr<int>() : nullptr;
  g.u0 = u0;
  g.len = len;
  g.shard = shard;
  g.w0 = consume ? w0 : u0;
  g.world = world;
  g.me = (int)me;
  g.copy_own = copy_own ? 1 : 0;
  launch_gemm(A, bp, Cout, (int)M, (int)N, (int)K, g, A.device());
  check_launch("gemm_gather_tc");
  return Cout;
}

namespace fsdp {

// Plain all-gather of a unit: this rank's buffer <- the owners' buffers,
// 16 bytes per thread per step, own range skipped unless `copy_own`.
__global__ void gather_kernel(const __nv_bfloat16* const* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                              int64_t u0, int64_t len, int64_t shard, int me, int copy_own) {
  const int64_t nv = len / 8;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = v * 8;
    const int owner = (int)(e / shard);
    if (owner == me && !copy_own) continue;
    *reinterpret_cast<uint4*>(dst + u0 + e) = *reinterpret_cast<const uint4*>(src[owner] + u0 + e);
  }
}

}  // namespace fsdp

// `src_ptrs[r] + u0 + e` is where owner r keeps unit element e (a caller can
// offset the pointers so the owners' parts come from a compact shard store).
void fsdp_gather(at::Tensor& flat, const at::Tensor& src_ptrs, int64_t u0, int64_t len, int64_t shard, int64_t me,
                 bool copy_own) {
  const at::cuda::CUDAGuard guard(flat.device());
  TORCH_CHECK(flat.is_cuda() && flat.scalar_type() == at::kBFloat16 && flat.is_contiguous() && aligned16(flat),
              "fsdp_gather: flat must be a contiguous bf16 CUDA buffer");
  TORCH_CHECK(u0 % 8 == 0 && len % 8 == 0 && shard % 8 == 0 && shard > 0 && u0 + len <= flat.numel(),
              "fsdp_gather: unit must be 8-element aligned and inside the buffer");
  TORCH_CHECK(shard * src_ptrs.numel() >= len, "fsdp_gather: shard layout");
  if (len == 0) return;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((len / 8 + 255) / 256, (int64_t)num_sms() * 8));
  fsdp::gather_kernel<<<blocks, 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16* const*>(src_ptrs.data_ptr<int64_t>()), (__nv_bfloat16*)flat.data_ptr(),
      u0, len, shard, (int)me, copy_own ? 1 : 0);
  check_launch("fsdp_gather");
}

}  // namespace tb
