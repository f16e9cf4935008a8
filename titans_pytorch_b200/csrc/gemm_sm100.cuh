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
// Warp roles per CTA (192 threads, or 320 for the epilogue-heavy modes; one
// CTA per SM, persistent):
//   warp 0      TMA producer (both CTAs)
//   warp 1      TMEM allocator (both CTAs, collectively); MMA issuer (leader)
//   warps 2-5   epilogue: thread = accumulator row (TMEM lane); two TMEM
//               accumulators of BN columns, so the epilogue of one tile
//               overlaps the next tile's main loop
//   warps 6-9   (SiLU' and SwiGLU-backward epilogues) a second set over the
//               same rows, taking every other column step
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
// Epilogues (a compile-time parameter of the kernel; every output is written once):
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
// tile-half to a workspace by TMA (the PARTIAL epilogue); a second kernel
// (splitk_reduce_kernel), spread over every SM, sums the partials of each
// output element in split order (a fixed order, so the result is
// deterministic) and applies the epilogue.  Nothing in the GEMM waits for
// another CTA.  Layout / epilogue pairs without a specialised kernel take the
// same route with one split.
//
// All mbarrier waits are bounded: a wait that runs out records an error code
// in the device error word and the CTA pair unwinds.
#pragma once

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
constexpr int BN_MAX = 256;   // tile columns: 256, or 128 for problems too small to fill the GPU
constexpr int BK = 64;        // k-slice per stage (128 bytes of bf16)
constexpr int NTHREADS = 192;
constexpr int EPI_WARP0 = 2;
constexpr int TM_COLS = 512;  // two accumulators of up to 256 columns
constexpr int STG_WARP = 16384;  // epilogue staging per warp: two sets of 8 KB

enum Mode : int {
  STORE = 0, ACCUM = 1, STORE_F32 = 2, RESID = 3, ACT = 4, ACT_GRAD = 5, ERR = 6, SWIGLU = 7, SWIGLU_BWD = 8,
  MEM_UPDATE = 9, PARTIAL = 10
};
enum : unsigned { ERR_TIMEOUT_PIPE = 50 };

struct Args {
  int M, N, K;
  int n_mt, n_nt, tiles, splits, kb_total, kb_per_split, items;
  int b_nstep, b_rstep;  // B-half row origin = nt * b_nstep + rank * b_rstep
  int mode, act, ffn_f, state_f32;
  int bn;  // tile columns (the kernel's BN; read by the split-K reduction)
  int cg;  // CTAs per tile (2: CTA pair, 256 rows; 1: one CTA, 128 rows)
  float scale;
  void* c;
  int64_t ldc;
  void* c2;
  int64_t ldc2;
  const float* gates;
  const void* r;
  int64_t ldr;
  const void* r2;
  int64_t ldr2;
  unsigned* err;
};

// Tensor maps of one launch.  Operands: a, b (128-byte swizzle, mainloop
// boxes).  Epilogue (32 x 32 boxes; bf16 with the 64-byte swizzle, fp32 with
// the 128-byte swizzle): c, c2 outputs, r, r2 inputs, ws the split-K partials
// ([items * 256, BN] fp32).  The SwiGLU backward reads g / u through r / r2
// and writes dg / du through c / c2 (each map covers its F columns, so
// edge blocks clip at F).  Unused maps repeat c.
struct Maps {
  CUtensorMap a, b, c, c2, r, r2, ws;
};

// Epilogue warp sets.  The input-gradient epilogues that read saved
// activations and compute a sigmoid and several products per output (SiLU'
// product, SwiGLU backward) outlast the short main loop of their K =
// model-width GEMMs; they run two sets of four epilogue warps over the same
// accumulator rows (TMEM lane quarters), each set taking every other 64-column
// step, and the main loop keeps three stages instead of five.  Measured on the
// MAG shapes (32768 x 3072, K = 768): SiLU' 0.195 -> 0.172 ms, SwiGLU
// backward 0.381 -> 0.353 ms; the SiLU forward epilogue (no input) was slower
// with the shallower main loop (0.150 -> 0.189 ms) and keeps one set.
template <int MODE>
constexpr int epi_sets() {
  return (MODE == SWIGLU_BWD || MODE == ACT_GRAD) ? 2 : 1;
}
template <int MODE>
constexpr int nthreads() {
  return 64 + 128 * epi_sets<MODE>();
}

template <int BN, int CG, int ES = 1>
struct Cfg {
  static constexpr int A_BYTES = HM * BK * 2;
  static constexpr int B_BYTES = (BN / CG) * BK * 2;  // this CTA's B rows
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NS = (ES == 1 ? 160 * 1024 : 96 * 1024) / STAGE;
  static constexpr int OFF_STG = NS * STAGE;
  static constexpr int OFF_BAR = OFF_STG + 4 * ES * STG_WARP;
  static constexpr int SMEM = OFF_BAR + 1024 + 1024;
  static_assert(NS >= 3, "main-loop stages");
};

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// Programmatic dependent launch: the kernel is launched so that it may start
// while the previous kernel on the stream is still running; wait() blocks
// until that kernel has completed and its writes are visible, trigger() lets
// the next kernel start its own prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
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
// The CTA-group generic forms (CG = 2: CTA pair, CG = 1: one CTA); every
// tcgen05 instruction of a kernel uses the same group.
template <int CG>
__device__ __forceinline__ void tmem_alloc_g(uint32_t* dst_smem, uint32_t ncols) {
  if constexpr (CG == 2) tmem_alloc2(dst_smem, ncols);
  else tc::tmem_alloc(dst_smem, ncols);
}
template <int CG>
__device__ __forceinline__ void tmem_relinquish_g() {
  if constexpr (CG == 2) tmem_relinquish2();
  else tc::tmem_relinquish();
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc_g(uint32_t taddr, uint32_t ncols) {
  if constexpr (CG == 2) tmem_dealloc2(taddr, ncols);
  else tc::tmem_dealloc(taddr, ncols);
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

template <int CG>
__device__ __forceinline__ void umma_g(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (CG == 2) umma2_bf16(tmem_d, adesc, bdesc, idesc, accumulate);
  else tc::umma_bf16(tmem_d, adesc, bdesc, idesc, accumulate);
}
template <int CG>
__device__ __forceinline__ void commit_g(uint64_t* bar) {
  if constexpr (CG == 2) umma2_commit_both(bar);
  else tc::umma_commit(bar);
}

// ------------------------------------------------------------------ epilogue blocks
// 2-D TMA load into this CTA's shared memory completing on a local barrier
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          tc::smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(tc::smem_addr(bar))
      : "memory");
}
// mainloop operand load: CG = 2 completes on the leader's barrier (cta_group::2
// form, shared::cluster address), CG = 1 on this CTA's own barrier
template <int CG>
__device__ __forceinline__ void op_load(void* dst, const CUtensorMap* map, uint32_t bar_addr, int c0, int c1) {
  if constexpr (CG == 2) {
    tma_load_2d_pair(dst, map, bar_addr, c0, c1);
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
            "r"(tc::smem_addr(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(bar_addr)
        : "memory");
  }
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


// ------------------------------------------------------------------ epilogue arithmetic
// The epilogues of the memory MLP and the SwiGLU evaluate a sigmoid per
// element; with MUFU (ex2 + rcp) and float->bf16 conversions all on the
// 16-per-clock pipe, they limited the short-K GEMMs.  Here each sigmoid takes
// one MUFU op (ex2) and the reciprocal 1 / (1 + e) runs on the FMA pipe:
// an initial estimate from integer subtraction off a magic constant (the
// reciprocal analogue of the well-known fast inverse square root bit trick,
// relative error below 12.5 %), refined by three Newton-Raphson steps
// r <- r (2 - d r), each of which squares the relative error (below 1e-7
// after three).  The argument is clamped at -87 so 1 + e stays finite.
__device__ __forceinline__ float rcp_nr(float d) {
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
  r = r * (2.f - d * r);
  r = r * (2.f - d * r);
  r = r * (2.f - d * r);
  return r;
}
__device__ __forceinline__ float sigmoid_nr(float x) { return rcp_nr(1.f + __expf(-fmaxf(x, -87.f))); }

// bf16 pair packing (one conversion per two values) and unpacking (shifts)
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// A row of 32 packed bf16 (16 words) into / out of a staging block (64-byte swizzle).
__device__ __forceinline__ void st_row_packed(uint8_t* blk, int r, const uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(blk + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}
__device__ __forceinline__ void ld_row_packed(const uint8_t* blk, int r, uint32_t (&w)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 u = *reinterpret_cast<const uint4*>(blk + r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
    w[4 * j] = u.x;
    w[4 * j + 1] = u.y;
    w[4 * j + 2] = u.z;
    w[4 * j + 3] = u.w;
  }
}

// ------------------------------------------------------------------ specialised epilogues
// Columns per epilogue step: 64 (128-byte bf16 rows, 128-byte swizzle) so
// every TMA row request moves a whole line; the SwiGLU forward (three
// output blocks per step) and the fp32 split-K partials use 32.
template <int MODE>
constexpr int step_cols() {
  return (MODE == SWIGLU || MODE == PARTIAL) ? 32 : 64;
}
// bytes of one 32-row block of the step (bf16, or fp32 for the partials)
template <int MODE>
constexpr int blk_bytes() {
  return MODE == PARTIAL ? 32 * 32 * 4 : 32 * step_cols<MODE>() * 2;
}
// bytes of input a MODE reads per step
template <int MODE>
constexpr uint32_t in_bytes() {
  return (MODE == RESID || MODE == ACCUM || MODE == ACT_GRAD || MODE == ERR)
             ? (uint32_t)blk_bytes<MODE>()
             : ((MODE == SWIGLU_BWD || MODE == MEM_UPDATE) ? 2u * blk_bytes<MODE>() : 0u);
}
// staging of one step (its input and output blocks)
template <int MODE>
constexpr int slot_bytes() {
  return MODE == SWIGLU ? 3 * blk_bytes<MODE>()
                       : ((MODE == ACT || MODE == SWIGLU_BWD || MODE == MEM_UPDATE) ? 2 : 1) * blk_bytes<MODE>();
}

// lane 0: loads the inputs of the block at output column n (rows row0..+31)
template <int MODE>
__device__ __forceinline__ void issue_in(const Maps& mp, int ffn_f, uint8_t* sb, int n, int row0, uint64_t* bar) {
  if constexpr (in_bytes<MODE>() > 0) {
    tc::mbar_expect_tx(bar, in_bytes<MODE>());
    tma_load_2d(sb, &mp.r, bar, n, row0);
    if constexpr (MODE == SWIGLU_BWD || MODE == MEM_UPDATE) tma_load_2d(sb + blk_bytes<MODE>(), &mp.r2, bar, n, row0);
  }
}

// Output column of epilogue step c of tile column nt, and the step count.
template <int MODE, int BN>
__device__ __forceinline__ int step_col(int nt, int c) {
  return MODE == SWIGLU ? nt * (BN / 2) + c * 32 : nt * BN + c * step_cols<MODE>();
}
template <int MODE, int BN>
__device__ __forceinline__ int step_count(const Args& p, int nt) {
  constexpr int SC = step_cols<MODE>();
  if constexpr (MODE == SWIGLU) return min(BN / 64, (p.ffn_f - nt * (BN / 2) + 31) / 32);
  else if constexpr (MODE == PARTIAL) return BN / 32;
  else return min(BN / SC, (p.N - nt * BN + SC - 1) / SC);
}

// 128-byte rows (64 bf16 = 32 words), 128-byte swizzle: chunk j at j ^ (r & 7)
__device__ __forceinline__ void st_row128(uint8_t* blk, int r, const uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(blk + r * 128 + ((j ^ (r & 7)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}
__device__ __forceinline__ void ld_row128(const uint8_t* blk, int r, uint32_t (&w)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 u = *reinterpret_cast<const uint4*>(blk + r * 128 + ((j ^ (r & 7)) << 4));
    w[4 * j] = u.x;
    w[4 * j + 1] = u.y;
    w[4 * j + 2] = u.z;
    w[4 * j + 3] = u.w;
  }
}

template <bool A_MN, bool B_MN, int MODE, int BN, int CG>
__global__ void __cluster_dims__(CG, 1, 1) __launch_bounds__(nthreads<MODE>(), 1)
    gemm2_kernel(const __grid_constant__ Maps mp, const Args p) {
  constexpr int ES = epi_sets<MODE>();
  using C = Cfg<BN, CG, ES>;
  constexpr int BMT = HM * CG;  // tile rows
  constexpr int NS = C::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* bar_empty = bar_full + NS;
  uint64_t* bar_acc_full = bar_empty + NS;
  uint64_t* bar_acc_empty = bar_acc_full + 2;
  uint64_t* bar_ld = bar_acc_empty + 2;  // 8 per epilogue warp (one per staging slot)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ld + 32 * ES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
  const int cid = blockIdx.x / CG, ncl = gridDim.x / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      tc::mbar_init(bar_full + s, 1);
      tc::mbar_init(bar_empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(bar_acc_full + b, 1);
      tc::mbar_init(bar_acc_empty + b, CG * 4 * ES);  // one arrival per epilogue warp of every CTA of the tile
    }
    for (int b = 0; b < 32 * ES; ++b) tc::mbar_init(bar_ld + b, 1);
    *abort_flag = 0;
    tc::mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_g<CG>(tmem_slot, TM_COLS);
    tmem_relinquish_g<CG>();
  }
  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive / complete_tx
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Everything above touched only this CTA's shared and tensor memory, so it
  // overlapped the previous kernel; global memory is read and written below.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      tc::tma_prefetch_desc(&mp.a);
      tc::tma_prefetch_desc(&mp.b);
      // the leader's full barriers (a single CTA's own)
      const uint32_t full0 = CG == 2 ? mapa(tc::smem_addr(bar_full), 0) : tc::smem_addr(bar_full);
      int it = 0;
      bool ok = true;
      for (int item = cid; ok && item < p.items; item += ncl) {
        int mt, nt, split;
        tile_of(p, item, mt, nt, split);
        const int kb0 = split * p.kb_per_split, kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int m0 = mt * BMT + (int)rank * HM;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NS;
          if (it >= NS && !tc::mbar_wait(bar_empty + s, ((it / NS) - 1) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          if (rank == 0) tc::mbar_expect_tx(bar_full + s, CG * C::STAGE);
          uint8_t* sa = smem + s * C::STAGE;
          uint8_t* sbm = sa + C::A_BYTES;
          const uint32_t fb = full0 + s * 8;
          const int k0 = kb * BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < HM / 64; ++j) op_load<CG>(sa + j * 8192, &mp.a, fb, m0 + 64 * j, k0);
          } else {
            op_load<CG>(sa, &mp.a, fb, k0, m0);
          }
          // B: the tile's two halves of BN / 2 rows (gate / up rows for the SwiGLU);
          // a CTA of a pair loads its own half, a single CTA both
#pragma unroll
          for (int hh = 0; hh < 2 / CG; ++hh) {
            const int half = CG == 2 ? (int)rank : hh;
            const int n0 = nt * p.b_nstep + half * p.b_rstep;
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                op_load<CG>(sbm + hh * (BN / 128) * 8192 + j * 8192, &mp.b, fb, n0 + 64 * j, k0);
            } else {
              op_load<CG>(sbm + hh * (BN / 2) * 128, &mp.b, fb, k0, n0);
            }
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
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BMT, BN, A_MN, B_MN);
      int it = 0, li = 0;
      bool ok = true;
      for (int item = cid; ok && item < p.items; item += ncl, ++li) {
        int mt, nt, split;
        tile_of(p, item, mt, nt, split);
        const int kb0 = split * p.kb_per_split, kb1 = min(p.kb_total, kb0 + p.kb_per_split);
        const int buf = li & 1;
        if (li >= 2 && !(CG == 2 ? mbar_wait_cluster(bar_acc_empty + buf, ((li >> 1) - 1) & 1, abort_flag, p.err)
                                  : tc::mbar_wait(bar_acc_empty + buf, ((li >> 1) - 1) & 1, abort_flag, p.err)))
          break;
        tc::tc_fence_after();
        const uint32_t d = tmem + buf * BN;
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
            umma_g<CG>(d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          commit_g<CG>(bar_empty + s);
        }
        if (ok) commit_g<CG>(bar_acc_full + buf);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5, and 6-9 with ES = 2)
    // Steps (column blocks) of this warp's tiles form one stream; the
    // staging buffer is a ring of NSLOT step slots, and the input blocks of
    // step k + NSLOT - 1 are requested right after step k's stores, across
    // tile boundaries, so load latency hides behind NSLOT - 1 steps.  With two
    // warp sets, set s takes steps s, s + 2, ... of every tile.
    constexpr int SLOT = slot_bytes<MODE>();
    constexpr int NSLOT = STG_WARP / SLOT;
    const int e = warp - EPI_WARP0;
    const int set = e >> 2;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* stg = smem + C::OFF_STG + e * STG_WARP;
    uint64_t* bl = bar_ld + 8 * e;
    uint32_t phase = 0;  // bit s: phase of slot s's load barrier
    const uint32_t acc_empty0 = CG == 2 ? mapa(tc::smem_addr(bar_acc_empty), 0) : tc::smem_addr(bar_acc_empty);
    const float scale = p.scale;
    const int ffn_f = p.ffn_f;
    // prefetch cursor (inputs only): next (item, step) of this warp whose inputs are requested
    int pf_item = cid, pf_c = set, pf_k = 0;
    auto prefetch_until = [&](int upto) {  // lane 0: request inputs of every own step < upto
      while (pf_k < upto && pf_item < p.items) {
        int pmt, pnt, psp;
        tile_of(p, pf_item, pmt, pnt, psp);
        const int ns = step_count<MODE, BN>(p, pnt);
        if (pf_c >= ns) {  // no (further) step of this warp in the tile
          pf_c = set;
          pf_item += ncl;
          continue;
        }
        const int prow0 = pmt * BMT + (int)rank * HM + q * 32;
        const int slot = pf_k % NSLOT;
        issue_in<MODE>(mp, ffn_f, stg + slot * SLOT, step_col<MODE, BN>(pnt, pf_c), prow0, bl + slot);
        ++pf_k;
        pf_c += ES;
        if (pf_c >= ns) {
          pf_c = set;
          pf_item += ncl;
        }
      }
    };
    if constexpr (in_bytes<MODE>() > 0) {
      if (lane == 0) prefetch_until(NSLOT - 1);
    }
    int li = 0, step = 0;
    bool ok = true;
    for (int item = cid; ok && item < p.items; item += ncl, ++li) {
      int mt, nt, split;
      tile_of(p, item, mt, nt, split);
      const int buf = li & 1;
      const int row0 = mt * BMT + (int)rank * HM + q * 32;
      const int nsteps = step_count<MODE, BN>(p, nt);
      if (!tc::mbar_wait(bar_acc_full + buf, (li >> 1) & 1, abort_flag, p.err)) break;
      tc::tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
      const int wrow = (item * CG + (int)rank) * HM + q * 32;  // PARTIAL: workspace rows
      if (set >= nsteps) {  // no step of this warp in the tile: release the accumulator at once
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty0 + buf * 8);
      }
      for (int c = set; c < nsteps; c += ES, ++step) {
        const int slot = step % NSLOT;
        uint8_t* sb = stg + slot * SLOT;
        const int n = step_col<MODE, BN>(nt, c);
        if constexpr (in_bytes<MODE>() == 0) {
          // the stores that last used this slot (NSLOT steps ago) have read it
          if (lane == 0) bulk_wait_read<NSLOT - 1>();
          __syncwarp();
        }
        constexpr int SC = step_cols<MODE>();
        float v[SC];
        float u[32];
        if constexpr (SC == 64) {
          float v1[32];
          tmem_row32(tbase + c * 64, *reinterpret_cast<float(*)[32]>(&v[0]));
          tmem_row32(tbase + c * 64 + 32, v1);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[32 + i] = v1[i];
        } else {
          tmem_row32(tbase + c * 32, *reinterpret_cast<float(*)[32]>(&v[0]));
        }
        if constexpr (MODE == SWIGLU) tmem_row32(tbase + BN / 2 + c * 32, u);
        if (c + ES >= nsteps) {  // this warp's last read of the accumulator: the MMA may reuse it
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acc_empty0 + buf * 8);
        }
        if constexpr (in_bytes<MODE>() > 0) {
          if (!tc::mbar_wait(bl + slot, (phase >> slot) & 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          phase ^= 1u << slot;
        }
        // ---- the epilogue math, thread = row `lane` of the block
        constexpr int BB = blk_bytes<MODE>();
        if constexpr (MODE == PARTIAL) {
          st_row_f32(sb, lane, *reinterpret_cast<float(*)[32]>(&v[0]));
        } else if constexpr (MODE == SWIGLU) {
          uint32_t gw[16], uw[16], hw[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            gw[i] = pack2(v[2 * i], v[2 * i + 1]);
            uw[i] = pack2(u[2 * i], u[2 * i + 1]);
            const float g0 = lo_bf(gw[i]), g1 = hi_bf(gw[i]);
            hw[i] = pack2(g0 * sigmoid_nr(g0) * lo_bf(uw[i]), g1 * sigmoid_nr(g1) * hi_bf(uw[i]));
          }
          st_row_packed(sb, lane, gw);
          st_row_packed(sb + BB, lane, uw);
          st_row_packed(sb + 2 * BB, lane, hw);
        } else {
          uint32_t w[32];  // 64 bf16 of this row
          if constexpr (MODE == STORE) {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = pack2(v[2 * i], v[2 * i + 1]);
          } else if constexpr (MODE == RESID || MODE == ACCUM) {
            ld_row128(sb, lane, w);
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = pack2(lo_bf(w[i]) + v[2 * i], hi_bf(w[i]) + v[2 * i + 1]);
          } else if constexpr (MODE == MEM_UPDATE) {
            // bf16 state: S' = bf16(eta S - theta G); W' = (1 - alpha) W + S'
            uint32_t sw[32];
            ld_row128(sb, lane, w);
            ld_row128(sb + BB, lane, sw);
            const float alpha = p.gates[0], theta = p.gates[1], eta = p.gates[2];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              sw[i] = pack2(eta * lo_bf(sw[i]) - theta * v[2 * i], eta * hi_bf(sw[i]) - theta * v[2 * i + 1]);
              w[i] = pack2((1.f - alpha) * lo_bf(w[i]) + lo_bf(sw[i]), (1.f - alpha) * hi_bf(w[i]) + hi_bf(sw[i]));
            }
            st_row128(sb + BB, lane, sw);
          } else if constexpr (MODE == ERR) {
            ld_row128(sb, lane, w);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              w[i] = pack2(scale * (v[2 * i] - lo_bf(w[i])), scale * (v[2 * i + 1] - hi_bf(w[i])));
          } else if constexpr (MODE == ACT_GRAD) {
            ld_row128(sb, lane, w);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float z0 = lo_bf(w[i]), z1 = hi_bf(w[i]);
              const float s0 = sigmoid_nr(z0), s1 = sigmoid_nr(z1);
              w[i] = pack2(v[2 * i] * s0 * (1.f + z0 * (1.f - s0)), v[2 * i + 1] * s1 * (1.f + z1 * (1.f - s1)));
            }
          } else if constexpr (MODE == ACT) {
            // z rounded to bf16 (stored for the backward); a = silu(z) from the rounded z
            uint32_t zw[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              zw[i] = pack2(v[2 * i], v[2 * i + 1]);
              const float z0 = lo_bf(zw[i]), z1 = hi_bf(zw[i]);
              w[i] = pack2(z0 * sigmoid_nr(z0), z1 * sigmoid_nr(z1));
            }
            st_row128(sb + BB, lane, zw);
          } else if constexpr (MODE == SWIGLU_BWD) {
            uint32_t uw[32];
            ld_row128(sb, lane, w);
            ld_row128(sb + BB, lane, uw);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float g0 = lo_bf(w[i]), g1 = hi_bf(w[i]), u0 = lo_bf(uw[i]), u1 = hi_bf(uw[i]);
              const float s0 = sigmoid_nr(g0), s1 = sigmoid_nr(g1);
              const float d0 = v[2 * i], d1 = v[2 * i + 1];
              w[i] = pack2(d0 * u0 * s0 * (1.f + g0 * (1.f - s0)), d1 * u1 * s1 * (1.f + g1 * (1.f - s1)));
              uw[i] = pack2(d0 * g0 * s0, d1 * g1 * s1);
            }
            st_row128(sb + BB, lane, uw);
          }
          st_row128(sb, lane, w);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (MODE == PARTIAL) {
            tma_store_2d(&mp.ws, sb, c * 32, wrow);
          } else if constexpr (MODE == SWIGLU) {
            tma_store_2d(&mp.c2, sb, n, row0);
            tma_store_2d(&mp.c2, sb + BB, ffn_f + n, row0);
            tma_store_2d(&mp.c, sb + 2 * BB, n, row0);
          } else if constexpr (MODE == SWIGLU_BWD || MODE == MEM_UPDATE) {
            tma_store_2d(&mp.c, sb, n, row0);
            tma_store_2d(&mp.c2, sb + BB, n, row0);
          } else if constexpr (MODE == ACT) {
            tma_store_2d(&mp.c, sb, n, row0);
            if (p.c2) tma_store_2d(&mp.c2, sb + BB, n, row0);
          } else {
            tma_store_2d(&mp.c, sb, n, row0);
          }
          bulk_commit();
          if constexpr (in_bytes<MODE>() > 0) {
            // the slot of step `step - 1` takes the inputs of step `step + NSLOT - 1`
            // once step - 1's stores have read it
            bulk_wait_read<1>();
            prefetch_until(step + NSLOT);
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0) bulk_wait_all();  // every store has landed before the CTA retires
    if constexpr (in_bytes<MODE>() > 0) {
      // inputs requested for steps that never ran (an abort) must land before the CTA retires
      if (lane == 0 && !ok) {
        volatile int keep = 0;
        for (int k = step; k < pf_k; ++k)
          tc::mbar_wait(bl + (k % NSLOT), (phase >> (k % NSLOT)) & 1, &keep, nullptr, 1ll << 27);
      }
    }
    __syncwarp();
  }

  tc::tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's MMAs / remote arrivals are done before TMEM and shared memory go away
  tc::tc_fence_after();
  if (warp == 1) tmem_dealloc_g<CG>(tmem, TM_COLS);
}

// Launch of one specialisation (defined in the per-layout translation units).
template <bool A_MN, bool B_MN, int MODE, int BN, int CG>
void launch_gemm2(const Maps& mp, const Args& a, cudaStream_t st);

// Grid: one tile group (CTA pair or CTA) per co-resident cluster slot, at most one per work item.
template <bool A_MN, bool B_MN, int MODE, int BN, int CG>
void launch_gemm2_impl(const Maps& mp, const Args& a, cudaStream_t st) {
  static int ncl_max = -1;
  using C = Cfg<BN, CG, epi_sets<MODE>()>;
  auto kern = gemm2_kernel<A_MN, B_MN, MODE, BN, CG>;
  if (ncl_max < 0) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CG * (num_sms() / CG));
    cfg.blockDim = dim3(nthreads<MODE>());
    cfg.dynamicSmemBytes = C::SMEM;
    int c = 0;
    if (cudaOccupancyMaxActiveClusters(&c, kern, &cfg) != cudaSuccess || c <= 0) {
      cudaGetLastError();
      c = num_sms() / CG;
    }
    ncl_max = std::min(c, num_sms() / CG);
  }
  const int ncl = std::min(a.items, ncl_max);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(CG * ncl);
  cfg.blockDim = dim3(nthreads<MODE>());
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, mp, a));
}

}  // namespace g2
}  // namespace tb
