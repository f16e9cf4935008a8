// Persistent 2-CTA tcgen05 GEMM for the training hot path, with fused
// epilogues and a deterministic split-K.
//
//   C[M, N] = sum_k A(m, k) * B(n, k)        (bf16 operands, fp32 in TMEM)
//
// Each operand is K-major (k contiguous: a row-major [rows, K] tensor) or
// MN-major (m / n contiguous: a row-major [K, rows] tensor), so one kernel
// covers the three GEMMs of a linear layer:
//   forward  y  = x W^T   : A = x  (K-major),  B = W (K-major)
//   dgrad    dx = dy W    : A = dy (K-major),  B = W (MN-major)
//   wgrad    dW = dy^T x  : A = dy (MN-major), B = x (MN-major), split-K over
//                           the token dimension, accumulated in place
//
// Tiles.  A cluster of two CTAs (a CTA pair on two SMs) owns a 256 x BN output
// tile.  CTA r loads A rows [128 r, 128 r + 128) of the tile and B rows
// [BN/2 r, BN/2 r + BN/2) into its own shared memory (TMA, 128-byte swizzle,
// no multicast); the leader CTA issues tcgen05.mma.cta_group::2 with M = 256,
// N = BN, which reads both CTAs' halves and writes rows 128 r.. of the
// accumulator into CTA r's tensor memory.  Both CTAs' loads complete on the
// leader's "full" barrier (cta_group::2 TMA form); MMA completion is
// multicast by tcgen05.commit to both CTAs' "empty" / "acc_full" barriers.
//
// Warp roles per CTA (192 threads, one CTA per SM, persistent):
//   warp 0      TMA producer (both CTAs)
//   warp 1      TMEM allocator (both CTAs, collectively); MMA issuer (leader)
//   warps 2-5   epilogue: thread = accumulator row (TMEM lane); two TMEM
//               accumulators of BN columns, so the epilogue of one tile
//               overlaps the next tile's main loop
//
// Epilogue data path.  Each epilogue warp owns 32 accumulator rows and works
// in 32 x 32 blocks: operands the epilogue reads (residual, saved
// activations, memory state, split-K partials) come in by TMA into a
// swizzled shared-memory block, each thread reads / writes its own row there
// (the swizzle keeps the 32 rows on distinct banks), and the results leave
// by TMA store.  Global traffic is therefore whole 128-byte lines; edge
// blocks are clipped (stores) and zero-filled (loads) by TMA itself.  Two
// block sets per warp alternate, so a block's store drains while the next
// block is computed.
//
// Epilogues (runtime mode; every output is written once):
//   STORE       C = bf16(acc)
//   ACCUM       C = bf16(C + acc)                     (weight gradients, beta = 1)
//   STORE_F32   C = acc (fp32)
//   RESID       C = bf16(R + acc)                     (residual add; R may alias C)
//   ACT         C2 = z = bf16(acc) (optional), C = act(z)
//   ACT_GRAD    C = bf16(bf16(acc) * act'(R))
//   ERR         C = bf16(scale * (bf16(acc) - R))     (associative-memory error)
//   SWIGLU      tile columns [0, BN/2) are gate rows, [BN/2, BN) up rows of the
//               stacked [Wg; Wu]: C2 = [g | u] (the gu buffer), C = silu(g) * u
//   SWIGLU_BWD  acc = dh: C = [dh * u * silu'(g) | dh * silu(g)] with [g | u] = R
//   MEM_UPDATE  acc = G (the full split-K sum): S' = eta S - theta G,
//               W' = (1 - alpha) W + S' with (alpha, theta, eta) read on the
//               device; R = W, R2 = S in, C = W', C2 = S' (state dtype)
//
// Split-K (work item = (tile, split)): each item stores its fp32 partial
// tile-half to a workspace, fences, and counts itself on the tile-half's
// counter; the item that brings the count to `splits` sums the partials in
// split order (the same order whoever arrives last, so the result is
// deterministic), runs the epilogue and resets the counter.  Nothing waits
// for another CTA, so no co-residency is needed.
//
// All mbarrier waits are bounded: a wait that runs out records an error code
// in the device error word and the CTA pair unwinds.
#include "tc_common.cuh"

namespace tb {

namespace attn_tc {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();
}  // namespace attn_tc
at::Tensor& tc_error_word(const at::Device& dev);

namespace g2 {

constexpr int HM = 128;       // accumulator rows per CTA
constexpr int BM = 2 * HM;    // tile rows per CTA pair
constexpr int BK = 64;        // k-slice per stage (128 bytes of bf16)
constexpr int NTHREADS = 192;
constexpr int EPI_WARP0 = 2;
constexpr int TM_COLS = 512;  // two accumulators of up to 256 columns

enum Mode : int {
  STORE = 0, ACCUM = 1, STORE_F32 = 2, RESID = 3, ACT = 4, ACT_GRAD = 5, ERR = 6, SWIGLU = 7, SWIGLU_BWD = 8,
  MEM_UPDATE = 9
};
enum : unsigned { ERR_TIMEOUT_PIPE = 50 };

struct Args {
  int M, N, K;
  int n_steps;           // 32-column epilogue steps per tile
  int n_mt, n_nt, tiles, splits, kb_total, kb_per_split, items;
  int b_nstep, b_rstep;  // B-half row origin = nt * b_nstep + rank * b_rstep
  int mode, act, ffn_f, state_f32;
  float scale;
  void* c;
  int64_t ldc;
  const void* r;
  int64_t ldr;
  void* c2;
  int64_t ldc2;
  const void* r2;
  int64_t ldr2;
  const float* gates;
  unsigned* cnt;
  unsigned* err;
};

// Tensor maps of one launch.  Operands: a, b (128-byte swizzle, mainloop
// boxes).  Epilogue (32 x 32 boxes; bf16 with the 64-byte swizzle, fp32 with
// the 128-byte swizzle): c, c2 outputs, r, r2 inputs, ws the split-K
// partials ([items * 256, BN] fp32).  Unused maps repeat c.
struct Maps {
  CUtensorMap a, b, c, c2, r, r2, ws;
};

constexpr int STG_WARP = 16384;  // epilogue staging per warp: two sets of 8 KB

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = HM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NS = (160 * 1024) / STAGE > 8 ? 8 : (160 * 1024) / STAGE;
  static constexpr int OFF_STG = NS * STAGE;
  static constexpr int OFF_BAR = OFF_STG + 4 * STG_WARP;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
};

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// shared::cluster address of the variable at local shared address `a` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(tc::smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait with cluster-scope acquire (arrivals come from the peer CTA)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  unsigned* err) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > (1ll << 31)) {
      *abort = 1;
      tc::set_error(err, ERR_TIMEOUT_PIPE);
      return false;
    }
  }
}
// 2-D tiled TMA load into this CTA's shared memory, completing on the
// barrier at shared::cluster address `mbar` (the leader CTA's)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t mbar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(tc::smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(mbar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc::smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma2_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at the same shared offset in both CTAs of the pair
// once every previously issued MMA of this thread has completed
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "{\n .reg .b16 m;\n mov.b16 m, 3;\n"
      " tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n}\n" ::"r"(
          tc::smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

// ------------------------------------------------------------------ epilogue blocks
// 2-D TMA load into this CTA's shared memory completing on a local barrier
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          tc::smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(tc::smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(map), "r"(c0),
               "r"(c1), "r"(tc::smem_addr(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;\n" ::: "memory"); }

// Row `r` of a 32 x 32 staging block (block base 1024-byte aligned).
// bf16: 64-byte rows, 16-byte chunk j at j ^ ((r >> 1) & 3) (64-byte swizzle);
// fp32: 128-byte rows, chunk j at j ^ (r & 7) (128-byte swizzle).
__device__ __forceinline__ void st_row_bf16(uint8_t* blk, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[8 * j + 2 * i], v[8 * j + 2 * i + 1]);
    *reinterpret_cast<uint4*>(blk + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) = u;
  }
}
__device__ __forceinline__ void ld_row_bf16(const uint8_t* blk, int r, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 u = *reinterpret_cast<const uint4*>(blk + r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[8 * j + 2 * i] = f.x;
      v[8 * j + 2 * i + 1] = f.y;
    }
  }
}
__device__ __forceinline__ void st_row_f32(uint8_t* blk, int r, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(blk + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
__device__ __forceinline__ void ld_row_f32(const uint8_t* blk, int r, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(blk + r * 128 + ((j ^ (r & 7)) << 4));
    v[4 * j] = f.x;
    v[4 * j + 1] = f.y;
    v[4 * j + 2] = f.z;
    v[4 * j + 3] = f.w;
  }
}
__device__ __forceinline__ void st_row(uint8_t* blk, int r, bool f32, const float (&v)[32]) {
  if (f32) st_row_f32(blk, r, v);
  else st_row_bf16(blk, r, v);
}
__device__ __forceinline__ void ld_row(const uint8_t* blk, int r, bool f32, float (&v)[32]) {
  if (f32) ld_row_f32(blk, r, v);
  else ld_row_bf16(blk, r, v);
}
__device__ __forceinline__ float rb(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Inputs the epilogue of `mode` reads for output columns [n, n + 32) of rows
// [row0, row0 + 32): issued by lane 0 into the slots of `sb`; returns the
// number of bytes the barrier expects (0: nothing to read).
__device__ __forceinline__ uint32_t epi_in_bytes(const Args& p) {
  const uint32_t blk = p.state_f32 ? 4096u : 2048u;
  switch (p.mode) {
    case ACCUM: case RESID: case ACT_GRAD: case ERR: return 2048u;
    case SWIGLU_BWD: return 4096u;
    case MEM_UPDATE: return 2 * blk;
    default: return 0u;
  }
}
__device__ __forceinline__ void epi_issue_inputs(const Args& p, const Maps& mp, uint8_t* sb, int n, int row0,
                                                 uint64_t* bar) {
  const uint32_t bytes = epi_in_bytes(p);
  if (bytes == 0) return;
  tc::mbar_expect_tx(bar, bytes);
  switch (p.mode) {
    case ACCUM: case RESID: case ACT_GRAD: case ERR:
      tma_load_2d(sb, &mp.r, bar, n, row0);
      break;
    case SWIGLU_BWD:
      tma_load_2d(sb, &mp.r, bar, n, row0);
      tma_load_2d(sb + 2048, &mp.r, bar, p.ffn_f + n, row0);
      break;
    case MEM_UPDATE: {
      const int blk = p.state_f32 ? 4096 : 2048;
      tma_load_2d(sb, &mp.r, bar, n, row0);
      tma_load_2d(sb + blk, &mp.r2, bar, n, row0);
      break;
    }
    default:
      break;
  }
}

// Computes the outputs of one 32-column block from the fp32 accumulator
// values `v` of this thread's row `r` (inputs already in the slots), writes
// them into the slots and (lane 0) issues their TMA stores + commit.
__device__ __forceinline__ void epi_finish(const Args& p, const Maps& mp, uint8_t* sb, int n, int row0, int r,
                                           float (&v)[32]) {
  float x[32];
  const bool f32s = p.state_f32 != 0;
  int nout = 1;
  switch (p.mode) {
    case STORE:
      st_row_bf16(sb, r, v);
      break;
    case STORE_F32:
      st_row_f32(sb, r, v);
      break;
    case ACCUM: case RESID:
      ld_row_bf16(sb, r, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] += v[i];
      st_row_bf16(sb, r, x);
      break;
    case ACT: {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = rb(v[i]);
      st_row_bf16(sb + 2048, r, v);  // z
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = act_f(p.act, v[i]);
      st_row_bf16(sb, r, x);
      nout = p.c2 ? 2 : 1;
      break;
    }
    case ACT_GRAD:
      ld_row_bf16(sb, r, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = rb(v[i]) * act_grad_f(p.act, x[i]);
      st_row_bf16(sb, r, x);
      break;
    case ERR:
      ld_row_bf16(sb, r, x);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = p.scale * (rb(v[i]) - x[i]);
      st_row_bf16(sb, r, x);
      break;
    case SWIGLU_BWD: {
      float u[32];
      ld_row_bf16(sb, r, x);
      ld_row_bf16(sb + 2048, r, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float d = rb(v[i]);
        const float dg = d * u[i] * silu_grad_(x[i]);
        u[i] = d * silu_(x[i]);
        x[i] = dg;
      }
      st_row_bf16(sb, r, x);
      st_row_bf16(sb + 2048, r, u);
      nout = 2;
      break;
    }
    case MEM_UPDATE: {
      const int blk = f32s ? 4096 : 2048;
      float sv[32];
      ld_row(sb, r, f32s, x);
      ld_row(sb + blk, r, f32s, sv);
      const float alpha = p.gates[0], theta = p.gates[1], eta = p.gates[2];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        // the momentum is rounded to the state dtype before it enters the
        // weight update (the reference builds S, then W, in that dtype)
        float sn = eta * sv[i] - theta * v[i];
        if (!f32s) sn = rb(sn);
        sv[i] = sn;
        x[i] = (1.f - alpha) * x[i] + sn;
      }
      st_row(sb, r, f32s, x);
      st_row(sb + blk, r, f32s, sv);
      nout = 2;
      break;
    }
    default:
      break;
  }
  tc::fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    switch (p.mode) {
      case SWIGLU_BWD:
        tma_store_2d(&mp.c, sb, n, row0);
        tma_store_2d(&mp.c, sb + 2048, p.ffn_f + n, row0);
        break;
      case MEM_UPDATE:
        tma_store_2d(&mp.c, sb, n, row0);
        tma_store_2d(&mp.c2, sb + (f32s ? 4096 : 2048), n, row0);
        break;
      case ACT:
        tma_store_2d(&mp.c, sb, n, row0);
        if (nout == 2) tma_store_2d(&mp.c2, sb + 2048, n, row0);
        break;
      default:
        tma_store_2d(&mp.c, sb, n, row0);
        break;
    }
    bulk_commit();
  }
}

__device__ __forceinline__ void tile_of(const Args& p, int item, int& mt, int& nt, int& split) {
  const int t = item / p.splits;
  split = item - t * p.splits;
  constexpr int G = 8;  // M-tiles per raster group: a 2048-row panel of A stays in L2 across the N tiles
  const int per_group = G * p.n_nt;
  const int grp = t / per_group, first = grp * G;
  const int gs = min(p.n_mt - first, G);
  const int w = t - grp * per_group;
  mt = first + w % gs;
  nt = w / gs;
}

__device__ __forceinline__ void tmem_row32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tc::tmem_ld32(taddr, r);
  tc::tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <bool A_MN, bool B_MN, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    gemm2_kernel(const __grid_constant__ Maps mp, const Args p) {
  using C = Cfg<BN>;
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_empty = bar_full + NS;
  uint64_t* bar_acc_full = bar_empty + NS;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_ld = bar_acc_empty + 2;  // 3 per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ld + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + s, 1);
      tc::mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_acc_full + b, 1);
      tc::mbar_init(bar_acc_empty + b, 2 * 4);  // one arrival per epilogue warp of both CTAs
    }
    for (int b = 0; b < 12; ++b) tc::mbar_init(bar_ld + b, 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, TM_COLS);
    tmem_relinquish2();
  }
  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive / complete_tx
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      tc::tma_prefetch_desc(&mp.a);
      tc::tma_prefetch_desc(&mp.b);
      const uint32_t full0 = mapa(tc::smem_addr(bar_full), 0);  // the leader's full barriers
      int it = 0;
      bool ok = true;
      for (int item = cid; ok && item < p.items; item += ncl) {
        int mt, nt, split;
        tile_of(p, item, mt, nt, split);
        const int kb0 = split * p.kb_per_split, kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int m0 = mt * BM + (int)rank * HM;
        const int n0 = nt * p.b_nstep + (int)rank * p.b_rstep;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NS;
          if (it >= NS && !tc::mbar_wait(bar_empty + s, ((it / NS) - 1) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          if (rank == 0) tc::mbar_expect_tx(bar_full + s, 2 * C::STAGE);
          uint8_t* sa = smem + s * C::STAGE;
          uint8_t* sbm = sa + C::A_BYTES;
          const uint32_t fb = full0 + s * 8;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < HM / 64; ++j) tma_load_2d_pair(sa + j * 8192, &mp.a, fb, m0 + 64 * j, k0);
          } else {
            tma_load_2d_pair(sa, &mp.a, fb, k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) tma_load_2d_pair(sbm + j * 8192, &mp.b, fb, n0 + 64 * j, k0);
          } else {
            tma_load_2d_pair(sbm, &mp.b, fb, k0, n0);
          }
        }
      }
      if (*abort_flag) {  // copies may still be landing: give them time before the CTA pair retires
        const long long t0 = clock64();
        while (clock64() - t0 < (1ll << 24)) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int it = 0, li = 0;
      bool ok = true;
      for (int item = cid; ok && item < p.items; item += ncl, ++li) {
        int mt, nt, split;
        tile_of(p, item, mt, nt, split);
        const int kb0 = split * p.kb_per_split, kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int buf = li & 1;
        if (li >= 2 && !mbar_wait_cluster(bar_acc_empty + buf, ((li >> 1) - 1) & 1, abort_flag, p.err)) break;
        tc::tc_fence_after();
        const uint32_t d = tmem + buf * 256;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NS;
          if (!tc::mbar_wait(bar_full + s, (it / NS) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t aA = tc::smem_addr(smem + s * C::STAGE), aB = aA + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? tc::sdesc_sw128(aA + k * 2048, 8192, 1024) : tc::sdesc_sw128(aA + 32 * k, 16, 1024);
            const uint64_t bd = B_MN ? tc::sdesc_sw128(aB + k * 2048, 8192, 1024) : tc::sdesc_sw128(aB + 32 * k, 16, 1024);
            umma2_bf16(d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma2_commit_both(bar_empty + s);
        }
        if (ok) umma2_commit_both(bar_acc_full + buf);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int e = warp - EPI_WARP0;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* stg = smem + C::OFF_STG + e * STG_WARP;
    uint64_t* bl = bar_ld + 3 * e;
    uint32_t ph0 = 0, ph1 = 0, ph2 = 0;  // phases of this warp's three load barriers
    const uint32_t acc_empty0 = mapa(tc::smem_addr(bar_acc_empty), 0);
    const bool swiglu = p.mode == SWIGLU;
    int li = 0, step = 0;
    bool ok = true;
    for (int item = cid; ok && item < p.items; item += ncl, ++li) {
      int mt, nt, split;
      tile_of(p, item, mt, nt, split);
      const int buf = li & 1;
      if (!tc::mbar_wait(bar_acc_full + buf, (li >> 1) & 1, abort_flag, p.err)) break;
      tc::tc_fence_after();
      const int row0 = mt * BM + (int)rank * HM + q * 32;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * 256;
      if (p.splits == 1) {
        const int nsteps = swiglu ? min(BN / 64, (p.ffn_f - nt * (BN / 2) + 31) / 32)
                                  : min(BN / 32, (p.N - nt * BN + 31) / 32);
        for (int c = 0; c < nsteps; ++c, ++step) {
          const int set = step & 1;
          uint8_t* sb = stg + set * 8192;
          uint64_t* bar = bl + set;
          if (lane == 0) bulk_wait_read<1>();  // the stores of two steps ago (same set) have read their blocks
          __syncwarp();
          if (swiglu) {
            const int j = nt * (BN / 2) + c * 32;
            float g[32], u[32];
            tmem_row32(tbase + c * 32, g);
            tmem_row32(tbase + BN / 2 + c * 32, u);
            if (c == nsteps - 1) {  // accumulator drained: the MMA may reuse it
              tc::tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(acc_empty0 + buf * 8);
            }
            float h[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              g[i] = rb(g[i]);
              u[i] = rb(u[i]);
              h[i] = silu_(g[i]) * u[i];
            }
            st_row_bf16(sb, lane, g);
            st_row_bf16(sb + 2048, lane, u);
            st_row_bf16(sb + 4096, lane, h);
            tc::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&mp.c2, sb, j, row0);
              tma_store_2d(&mp.c2, sb + 2048, p.ffn_f + j, row0);
              tma_store_2d(&mp.c, sb + 4096, j, row0);
              bulk_commit();
            }
          } else {
            const int n = nt * BN + c * 32;
            const bool has_in = epi_in_bytes(p) != 0;
            if (has_in && lane == 0) epi_issue_inputs(p, mp, sb, n, row0, bar);
            float v[32];
            tmem_row32(tbase + c * 32, v);
            if (c == nsteps - 1) {
              tc::tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(acc_empty0 + buf * 8);
            }
            if (has_in) {
              uint32_t& ph = set ? ph1 : ph0;
              if (!tc::mbar_wait(bar, ph, abort_flag, p.err)) {
                ok = false;
                break;
              }
              ph ^= 1;
            }
            epi_finish(p, mp, sb, n, row0, lane, v);
          }
        }
      } else {
        // ---- split-K: this item's fp32 partial -> workspace rows (item, rank, q)
        const int tile = item / p.splits;
        const int wrow = (item * 2 + (int)rank) * HM + q * 32;
        for (int c = 0; c < BN / 32; ++c, ++step) {
          uint8_t* sb = stg + (step & 1) * 8192;
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
          float v[32];
          tmem_row32(tbase + c * 32, v);
          if (c == BN / 32 - 1) {
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty0 + buf * 8);
          }
          st_row_f32(sb, lane, v);
          tc::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mp.ws, sb, c * 32, wrow);
            bulk_commit();
          }
        }
        // partial complete and visible before it is counted
        if (lane == 0) {
          bulk_wait_all();
          fence_proxy_async_global();
          __threadfence();
        }
        __syncwarp();
        epi_bar();
        if (threadIdx.x == EPI_WARP0 * 32) {
          unsigned* cnt = p.cnt + tile * 2 + rank;
          const unsigned prev = atomicAdd(cnt, 1u);
          const bool last = prev == (unsigned)(p.splits - 1);
          if (last) atomicExch(cnt, 0u);  // ready for the next launch
          *last_flag = last ? 1 : 0;
        }
        epi_bar();
        if (*last_flag) {
          // ---- the last item of the tile sums the partials in split order
          if (lane == 0) {
            __threadfence();
            fence_proxy_async_global();
          }
          __syncwarp();
          const int nsteps = min(BN / 32, (p.N - nt * BN + 31) / 32);
          const int prow0 = (tile * p.splits * 2 + (int)rank) * HM + q * 32;  // split 0's rows
          const int pstride = 2 * HM;                                         // rows between splits
          uint8_t* ob = stg + 8192;  // output / input slots of the reduced block
          for (int c = 0; c < nsteps && ok; ++c) {
            const int n = nt * BN + c * 32;
            if (lane == 0) bulk_wait_read<0>();  // previous block's stores have read the output slots
            __syncwarp();
            const bool has_in = epi_in_bytes(p) != 0;
            if (has_in && lane == 0) epi_issue_inputs(p, mp, ob, n, row0, bl + 2);
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[i] = 0.f;
            if (lane == 0) {
              tc::mbar_expect_tx(bl + 0, 4096);
              tma_load_2d(stg, &mp.ws, bl + 0, c * 32, prow0);
            }
            for (int sp = 0; sp < p.splits; ++sp) {
              const int pb = sp & 1;
              if (sp + 1 < p.splits && lane == 0) {
                tc::mbar_expect_tx(bl + (pb ^ 1), 4096);
                tma_load_2d(stg + (pb ^ 1) * 4096, &mp.ws, bl + (pb ^ 1), c * 32, prow0 + (sp + 1) * pstride);
              }
              uint32_t& ph = pb ? ph1 : ph0;
              if (!tc::mbar_wait(bl + pb, ph, abort_flag, p.err)) {
                ok = false;
                break;
              }
              ph ^= 1;
              float v[32];
              ld_row_f32(stg + pb * 4096, lane, v);
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] += v[i];
              __syncwarp();  // every lane has read the buffer before it is refilled
            }
            if (!ok) break;
            if (has_in) {
              if (!tc::mbar_wait(bl + 2, ph2, abort_flag, p.err)) {
                ok = false;
                break;
              }
              ph2 ^= 1;
            }
            epi_finish(p, mp, ob, n, row0, lane, acc);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // every store has landed before the CTA retires
    __syncwarp();
  }

  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's MMAs / remote arrivals are done before TMEM and shared memory go away
  tc::tc_fence_after();
  if (warp == 1) tmem_dealloc2(tmem, TM_COLS);
}

}  // namespace g2

namespace {

// 2-D tensor map over a row-major [rows, inner] matrix with leading dimension
// `ld` (elements); box = box_inner x box_rows.
CUtensorMap make_map_2d(const void* base, CUtensorMapDataType dt, int esize, uint64_t inner, uint64_t rows,
                        uint64_t ld, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)esize};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = attn_tc::encode_tiled_fn()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "gemm_sm100: cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}
CUtensorMap operand_map(const at::Tensor& t, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  return make_map_2d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, rows, t.stride(0), 64, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}
// epilogue block map: 32 x 32 elements of a [rows, cols] bf16 / fp32 matrix
CUtensorMap epi_map(const at::Tensor& t, uint64_t cols, uint64_t rows) {
  const bool f32 = t.scalar_type() == at::kFloat;
  return make_map_2d(t.data_ptr(), f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                     f32 ? 4 : 2, cols, rows, t.stride(0), 32, 32,
                     f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

template <bool A_MN, bool B_MN, int BN>
int max_clusters() {
  static int n = -1;
  if (n < 0) {
    using C = g2::Cfg<BN>;
    auto kern = g2::gemm2_kernel<A_MN, B_MN, BN>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(g2::NTHREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess || c <= 0) {
      cudaGetLastError();
      c = num_sms() / 2;
    }
    n = std::min(c, num_sms() / 2);
  }
  return n;
}

template <bool A_MN, bool B_MN, int BN>
void launch(const g2::Maps& mp, const g2::Args& a) {
  using C = g2::Cfg<BN>;
  const int ncl = std::min(a.items, max_clusters<A_MN, B_MN, BN>());
  g2::gemm2_kernel<A_MN, B_MN, BN><<<2 * ncl, g2::NTHREADS, C::SMEM, stream()>>>(mp, a);
}

// Split-K count for `tiles` output tiles over a K of `kb` 64-wide slices on
// `ncl` CTA pairs: minimises (waves x slices per split) plus a cost per split
// for writing and summing its partial, with at least 8 slices per split.
int choose_splits(int tiles, int kb, int ncl) {
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= 32; ++s) {
    if (s > 1 && kb / s < 8) break;
    const int per = (kb + s - 1) / s;
    if ((kb + per - 1) / per != s) continue;
    const int items = tiles * s;
    const int waves = (items + ncl - 1) / ncl;
    const double cost = (double)waves * per + (s > 1 ? 3.0 * s : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

void check_mat(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1, "gemm_sm100: ", what,
              " must be a 2-D CUDA tensor with a contiguous last dim");
  TORCH_CHECK((uintptr_t)t.data_ptr() % 16 == 0 && (t.stride(0) * t.element_size()) % 16 == 0, "gemm_sm100: ",
              what, " must be 16-byte aligned with a 16-byte row pitch");
}

}  // namespace

// C[M, N] = A . B with A given K-major ([M, K]) or MN-major ([K, M]), B
// K-major ([N, K]) or MN-major ([K, N]); fused epilogue `mode` (g2::Mode).
// `splits` <= 0 picks a split-K count (modes that allow it), 1 disables it.
void gemm_sm100(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t M, int64_t N, int64_t K,
                int64_t mode, const at::Tensor& Cout, const c10::optional<at::Tensor>& R,
                const c10::optional<at::Tensor>& C2, const c10::optional<at::Tensor>& R2,
                const c10::optional<at::Tensor>& gates, double scale, int64_t act, int64_t ffn_f, int64_t splits) {
  using namespace g2;
  const at::cuda::CUDAGuard guard(A.device());
  check_mat(A, "A");
  check_mat(B, "B");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_sm100: bf16 operands");
  TORCH_CHECK(M > 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
              "gemm_sm100: bad sizes");
  TORCH_CHECK(N % 8 == 0, "gemm_sm100: N must be a multiple of 8");
  TORCH_CHECK(mode >= STORE && mode <= MEM_UPDATE, "gemm_sm100: unknown epilogue");
  if (a_mn) {
    TORCH_CHECK(A.size(0) >= K && A.size(1) >= M, "gemm_sm100: A [K, M]");
  } else {
    TORCH_CHECK(A.size(0) >= M && A.size(1) >= K, "gemm_sm100: A [M, K]");
  }
  const bool swiglu = mode == SWIGLU;
  if (swiglu) {
    TORCH_CHECK(!b_mn && ffn_f > 0 && ffn_f % 32 == 0 && N == 2 * ffn_f && B.size(0) >= 2 * ffn_f &&
                    B.size(1) >= K,
                "gemm_sm100: SWIGLU needs the stacked K-major [Wg; Wu], N = 2F and F a multiple of 32");
  } else if (b_mn) {
    TORCH_CHECK(B.size(0) >= K && B.size(1) >= N, "gemm_sm100: B [K, N]");
  } else {
    TORCH_CHECK(B.size(0) >= N && B.size(1) >= K, "gemm_sm100: B [N, K]");
  }
  if (mode == SWIGLU_BWD) TORCH_CHECK(N % 32 == 0, "gemm_sm100: SWIGLU_BWD needs F a multiple of 32");
  check_mat(Cout, "C");
  if (mode == STORE_F32) {
    TORCH_CHECK(Cout.scalar_type() == at::kFloat, "gemm_sm100: STORE_F32 writes fp32");
  } else if (mode == MEM_UPDATE) {
    TORCH_CHECK(Cout.scalar_type() == at::kFloat || Cout.scalar_type() == at::kBFloat16,
                "gemm_sm100: memory state must be fp32 or bf16");
  } else {
    TORCH_CHECK(Cout.scalar_type() == at::kBFloat16, "gemm_sm100: bf16 output");
  }
  const int64_t c_cols = swiglu ? ffn_f : (mode == SWIGLU_BWD ? 2 * N : N);
  TORCH_CHECK(Cout.size(0) >= M && Cout.size(1) >= c_cols, "gemm_sm100: output too small");
  const bool needs_r = mode == RESID || mode == ACT_GRAD || mode == ERR || mode == SWIGLU_BWD || mode == MEM_UPDATE;
  if (needs_r) {
    TORCH_CHECK(R.has_value(), "gemm_sm100: mode needs R");
    check_mat(*R, "R");
    TORCH_CHECK(R->size(0) >= M && R->size(1) >= (mode == SWIGLU_BWD ? 2 * N : N), "gemm_sm100: R too small");
    TORCH_CHECK(R->scalar_type() == Cout.scalar_type(), "gemm_sm100: R dtype");
  }
  if (mode == SWIGLU || mode == MEM_UPDATE) TORCH_CHECK(C2.has_value(), "gemm_sm100: mode needs C2");
  const int64_t c2_cols = swiglu ? 2 * ffn_f : N;
  if (C2.has_value()) {
    check_mat(*C2, "C2");
    TORCH_CHECK(C2->scalar_type() == Cout.scalar_type() && C2->size(0) >= M && C2->size(1) >= c2_cols,
                "gemm_sm100: C2 shape / dtype");
  }
  if (mode == MEM_UPDATE) {
    TORCH_CHECK(R2.has_value() && gates.has_value(), "gemm_sm100: MEM_UPDATE needs R2 and gates");
    check_mat(*R2, "R2");
    TORCH_CHECK(R2->scalar_type() == Cout.scalar_type() && R2->size(0) >= M && R2->size(1) >= N,
                "gemm_sm100: R2 shape / dtype");
    TORCH_CHECK(gates->is_cuda() && gates->scalar_type() == at::kFloat && gates->numel() >= 3,
                "gemm_sm100: gates float[3] on the device");
  }

  constexpr int BN = 256;
  Args a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.n_mt = (int)((M + BM - 1) / BM);
  a.n_nt = swiglu ? (int)((ffn_f + BN / 2 - 1) / (BN / 2)) : (int)((N + BN - 1) / BN);
  a.tiles = a.n_mt * a.n_nt;
  a.kb_total = (int)((K + BK - 1) / BK);
  int ncl = 0;
  if (a_mn && b_mn) ncl = max_clusters<true, true, BN>();
  else if (a_mn) ncl = max_clusters<true, false, BN>();
  else if (b_mn) ncl = max_clusters<false, true, BN>();
  else ncl = max_clusters<false, false, BN>();
  const bool split_ok = !swiglu;
  int s = (int)splits;
  if (s <= 0) s = split_ok ? choose_splits(a.tiles, a.kb_total, ncl) : 1;
  TORCH_CHECK(s == 1 || split_ok, "gemm_sm100: this epilogue does not take split-K");
  s = std::max(1, std::min(s, a.kb_total));
  a.kb_per_split = (a.kb_total + s - 1) / s;
  a.splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  a.items = a.tiles * a.splits;
  a.b_nstep = swiglu ? BN / 2 : BN;
  a.b_rstep = swiglu ? (int)ffn_f : BN / 2;
  a.mode = (int)mode;
  a.act = (int)act;
  a.ffn_f = (int)(swiglu ? ffn_f : (mode == SWIGLU_BWD ? N : 0));
  a.state_f32 = (mode == MEM_UPDATE && Cout.scalar_type() == at::kFloat) ? 1 : 0;
  a.scale = (float)scale;
  a.c = Cout.data_ptr();
  a.ldc = Cout.stride(0);
  if (C2.has_value()) {
    a.c2 = C2->data_ptr();
    a.ldc2 = C2->stride(0);
  }
  if (gates.has_value()) a.gates = gates->data_ptr<float>();
  a.err = (unsigned*)tc_error_word(A.device()).data_ptr<int>();

  Maps mp;
  mp.a = a_mn ? operand_map(A, M, K, 64) : operand_map(A, K, M, HM);
  const int64_t b_rows = swiglu ? 2 * ffn_f : N;
  mp.b = b_mn ? operand_map(B, N, K, 64) : operand_map(B, K, b_rows, BN / 2);
  mp.c = epi_map(Cout, c_cols, M);
  mp.c2 = C2.has_value() ? epi_map(*C2, c2_cols, M) : mp.c;
  if (mode == ACCUM) mp.r = mp.c;
  else mp.r = needs_r ? epi_map(*R, mode == SWIGLU_BWD ? 2 * N : N, M) : mp.c;
  mp.r2 = R2.has_value() ? epi_map(*R2, N, M) : mp.c;
  mp.ws = mp.c;
  at::Tensor ws;
  if (a.splits > 1) {
    // fp32 partial tile-halves [items * 256, BN], then one counter per
    // tile-half (zeroed here; the last item of a tile resets its counter)
    const int64_t part = (int64_t)a.items * 2 * HM * BN;
    ws = at::empty({part + 2 * (int64_t)a.tiles + 64}, A.options().dtype(at::kFloat));
    a.cnt = reinterpret_cast<unsigned*>(ws.data_ptr<float>() + part);
    C10_CUDA_CHECK(cudaMemsetAsync(a.cnt, 0, 2 * (size_t)a.tiles * sizeof(unsigned), stream()));
    at::Tensor wsv = ws.narrow(0, 0, part).view({(int64_t)a.items * 2 * HM, BN});
    mp.ws = epi_map(wsv, BN, (uint64_t)a.items * 2 * HM);
  }
  if (a_mn && b_mn) launch<true, true, BN>(mp, a);
  else if (a_mn) launch<true, false, BN>(mp, a);
  else if (b_mn) launch<false, true, BN>(mp, a);
  else launch<false, false, BN>(mp, a);
  check_launch("gemm_sm100");
}

}  // namespace tb
