// Host side of the 2-CTA tcgen05 GEMM (kernels in gemm_sm100.cuh, specialised
// per operand layout and tile shape in gemm_sm100_k2.cu / _k2n.cu / _k1.cu / _mn.cu) and the split-K
// reduction kernel.
#include "gemm_sm100.cuh"

namespace tb {
namespace g2 {

// ------------------------------------------------------------------ split-K reduction
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void ld8f(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void st8f(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Epilogue of 8 consecutive columns [n, n + 8) of row m (inside M x N) from
// their fp32 sums, for the modes that take split-K.
__device__ __forceinline__ void epi8(const Args& p, int64_t m, int n, const float (&v)[8]) {
  float o[8], x[8];
  switch (p.mode) {
    case STORE:
      st8((__nv_bfloat16*)p.c + m * p.ldc + n, v);
      break;
    case STORE_F32:
      st8f((float*)p.c + m * p.ldc + n, v);
      break;
    case ACCUM: case RESID: {
      const __nv_bfloat16* src = p.mode == ACCUM ? (const __nv_bfloat16*)p.c + m * p.ldc + n
                                                 : (const __nv_bfloat16*)p.r + m * p.ldr + n;
      ld8(src, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = x[i] + v[i];
      st8((__nv_bfloat16*)p.c + m * p.ldc + n, o);
      break;
    }
    case ACT:
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = rb(v[i]);
        o[i] = act_f(p.act, x[i]);
      }
      if (p.c2) st8((__nv_bfloat16*)p.c2 + m * p.ldc2 + n, x);
      st8((__nv_bfloat16*)p.c + m * p.ldc + n, o);
      break;
    case ACT_GRAD:
      ld8((const __nv_bfloat16*)p.r + m * p.ldr + n, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rb(v[i]) * act_grad_f(p.act, x[i]);
      st8((__nv_bfloat16*)p.c + m * p.ldc + n, o);
      break;
    case ERR:
      ld8((const __nv_bfloat16*)p.r + m * p.ldr + n, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = p.scale * (rb(v[i]) - x[i]);
      st8((__nv_bfloat16*)p.c + m * p.ldc + n, o);
      break;
    case MEM_UPDATE: {
      float w[8], sv[8];
      const float alpha = p.gates[0], theta = p.gates[1], eta = p.gates[2];
      if (p.state_f32) {
        ld8f((const float*)p.r + m * p.ldr + n, w);
        ld8f((const float*)p.r2 + m * p.ldr2 + n, sv);
      } else {
        ld8((const __nv_bfloat16*)p.r + m * p.ldr + n, w);
        ld8((const __nv_bfloat16*)p.r2 + m * p.ldr2 + n, sv);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float sn = eta * sv[i] - theta * v[i];
        if (!p.state_f32) sn = rb(sn);
        sv[i] = sn;
        o[i] = (1.f - alpha) * w[i] + sn;
      }
      if (p.state_f32) {
        st8f((float*)p.c2 + m * p.ldc2 + n, sv);
        st8f((float*)p.c + m * p.ldc + n, o);
      } else {
        st8((__nv_bfloat16*)p.c2 + m * p.ldc2 + n, sv);
        st8((__nv_bfloat16*)p.c + m * p.ldc + n, o);
      }
      break;
    }
    default:
      break;
  }
}

// One thread per 8 columns of one accumulator row: sums the `splits`
// partials (split 0 first) from the workspace and runs the epilogue.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, const Args p) {
  pdl_wait();  // launched as a programmatic dependent of the GEMM that wrote the partials
  pdl_trigger();
  const int BN = p.bn, CH = BN / 8, BMT = HM * p.cg;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)p.tiles * BMT * CH;
  if (idx >= total) return;
  const int ch = (int)(idx % CH);
  const int row = (int)((idx / CH) % BMT);  // row inside the tile (CTA of the pair = row / 128)
  const int t = (int)(idx / ((int64_t)CH * BMT));
  int mt, nt, split;
  tile_of(p, t * p.splits, mt, nt, split);
  const int64_t m = (int64_t)mt * BMT + row;
  const int n = nt * BN + ch * 8;
  if (m >= p.M || n >= p.N) return;
  const int half = row / HM, r_in = row % HM;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const int64_t wrow = ((int64_t)(t * p.splits + s) * p.cg + half) * HM + r_in;
    float v[8];
    ld8f(ws + wrow * BN + ch * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  epi8(p, m, n, acc);
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
// epilogue block map of a [rows, cols] bf16 / fp32 matrix: 32 rows x `box_cols`
// (bf16: 32 columns with the 64-byte swizzle or 64 with the 128-byte one;
// fp32: 32 columns, 128-byte swizzle)
CUtensorMap epi_map(const at::Tensor& t, uint64_t cols, uint64_t rows, uint32_t box_cols = 32) {
  const bool f32 = t.scalar_type() == at::kFloat;
  const bool wide = f32 || box_cols == 64;
  return make_map_2d(t.data_ptr(), f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                     f32 ? 4 : 2, cols, rows, t.stride(0), f32 ? 32 : box_cols, 32,
                     wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// Split-K count for `tiles` output tiles over a K of `kb` 64-wide slices on
// `ncl` CTA pairs.  Cost in units of one 64-wide slice of a tile's MMAs:
// waves x slices per split, plus, whenever partials are written (split-K, or
// an epilogue that always goes through them), about 12 units per work item
// for the fp32 partial and its share of the reduction, and 20 units for the
// reduction kernel's launch and ramp.  At least 8 slices per split.
int choose_splits(int tiles, int kb, int ncl, bool partial_anyway) {
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= 32; ++s) {
    if (s > 1 && kb / s < 8) break;
    const int per = (kb + s - 1) / s;
    if ((kb + per - 1) / per != s) continue;
    const int items = tiles * s;
    const int waves = (items + ncl - 1) / ncl;
    double cost = (double)waves * per;
    if (s > 1 || partial_anyway) cost += 12.0 * waves + 12.0 * items / ncl + 20.0;
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
  if (mode == SWIGLU_BWD) TORCH_CHECK(N % 8 == 0, "gemm_sm100: SWIGLU_BWD needs F a multiple of 8");
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

  Args a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;

  a.kb_total = (int)((K + BK - 1) / BK);
  const int ncl = std::max(1, num_sms() / 2);
  const bool state_f32_req = mode == MEM_UPDATE && Cout.scalar_type() == at::kFloat;
  // Tile shape: 256 x 256 on CTA pairs; 256 x 128 on CTA pairs when the
  // 256-wide tiles would not fill one wave of pairs (weight gradients fill
  // the GPU with split-K instead); 128 x 128 on single CTAs for at most 128
  // rows (a pair's second half would be empty).  A single CTA streaming
  // 128 x 128 x 64 per stage is bound by shared-memory bandwidth at about
  // half the tensor rate, so it is not used where pairs fit.
  const auto n_tiles = [&](int bm, int bn) {
    return (int)((M + bm - 1) / bm) *
           (swiglu ? (int)((ffn_f + bn / 2 - 1) / (bn / 2)) : (int)((N + bn - 1) / bn));
  };
  int BN = 256, CG = 2;
  if (M <= HM) {
    BN = 128;
    CG = 1;
  } else if (!(a_mn && b_mn) && n_tiles(256, 256) < ncl && n_tiles(256, 128) > n_tiles(256, 256)) {
    BN = 128;
  }
  a.bn = BN;
  a.cg = CG;
  a.n_mt = (int)((M + HM * CG - 1) / (HM * CG));
  a.n_nt = swiglu ? (int)((ffn_f + BN / 2 - 1) / (BN / 2)) : (int)((N + BN - 1) / BN);
  a.tiles = a.n_mt * a.n_nt;
  const int ngroups = std::max(1, num_sms() / CG);  // tile groups that run at once
  const bool split_ok = !swiglu;
  int s = (int)splits;
  const bool partial_anyway =
      !(mode == STORE || mode == RESID || mode == ACT || mode == ERR || mode == ACT_GRAD || mode == SWIGLU ||
        mode == SWIGLU_BWD || (a_mn && b_mn && (mode == ACCUM || (mode == MEM_UPDATE && !state_f32_req))));
  if (s <= 0) s = split_ok ? choose_splits(a.tiles, a.kb_total, ngroups, partial_anyway) : 1;
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

  if (R.has_value()) {
    a.r = R->data_ptr();
    a.ldr = R->stride(0);
  }
  if (mode == ACCUM) {
    a.r = a.c;
    a.ldr = a.ldc;
  }
  if (R2.has_value()) {
    a.r2 = R2->data_ptr();
    a.ldr2 = R2->stride(0);
  }
  // kernel: a specialised epilogue, or fp32 partials + the reduction kernel
  const bool silu = act == ACT_SILU;
  int kmode = PARTIAL;
  if (a.splits == 1) {
    if (!a_mn && !b_mn &&
        (mode == STORE || mode == RESID || (mode == ACT && silu) || mode == ERR || mode == SWIGLU))
      kmode = (int)mode;
    else if (!a_mn && b_mn && (mode == STORE || (mode == ACT_GRAD && silu) || mode == SWIGLU_BWD))
      kmode = (int)mode;
    else if (a_mn && b_mn && (mode == ACCUM || (mode == MEM_UPDATE && !a.state_f32)))
      kmode = (int)mode;
    else if (mode == STORE)
      kmode = STORE;
  }
  TORCH_CHECK(kmode != PARTIAL || (mode != SWIGLU && mode != SWIGLU_BWD),
              "gemm_sm100: SwiGLU epilogues need K-major A (and B for the forward)");
  // epilogue maps: 64-column blocks, except the SwiGLU forward's 32
  const uint32_t bc = kmode == SWIGLU ? 32 : 64;
  mp.c = epi_map(Cout, c_cols, M, bc);
  mp.c2 = C2.has_value() ? epi_map(*C2, c2_cols, M, bc) : mp.c;
  mp.r = needs_r ? epi_map(*R, N, M, bc) : mp.c;
  if (mode == ACCUM) mp.r = mp.c;
  mp.r2 = (mode == MEM_UPDATE && !a.state_f32) ? epi_map(*R2, N, M, bc) : mp.c;
  if (mode == SWIGLU_BWD) {  // [dg | du] and [g | u] as two F-column halves each
    mp.c = epi_map(Cout, N, M, bc);
    mp.c2 = epi_map(Cout.narrow(1, N, N), N, M, bc);
    mp.r2 = epi_map(R->narrow(1, N, N), N, M, bc);
  }
  mp.ws = mp.c;
  at::Tensor ws;
  if (kmode == PARTIAL) {
    // fp32 partials, 128 rows per CTA of each work item: [items * CG * 128, BN]
    ws = at::empty({(int64_t)a.items * CG * HM, BN}, A.options().dtype(at::kFloat));
    mp.ws = epi_map(ws, BN, (uint64_t)a.items * CG * HM);
  }
  cudaStream_t st = stream();
#define TB_G2(AM, BMN, MD)                                                          \
  if (a_mn == AM && b_mn == BMN && kmode == MD) {                                     \
    if (CG == 1) launch_gemm2<AM, BMN, MD, 128, 1>(mp, a, st);                        \
    else if (BN == 256) launch_gemm2<AM, BMN, MD, 256, 2>(mp, a, st);                 \
    else launch_gemm2<AM, BMN, MD, 128, 2>(mp, a, st);                                \
    goto launched;                                                                    \
  }
  TB_G2(false, false, STORE) TB_G2(false, false, RESID) TB_G2(false, false, ACT) TB_G2(false, false, ERR)
  TB_G2(false, false, SWIGLU) TB_G2(false, false, PARTIAL)
  TB_G2(false, true, STORE) TB_G2(false, true, ACT_GRAD) TB_G2(false, true, SWIGLU_BWD) TB_G2(false, true, PARTIAL)
  TB_G2(true, true, STORE) TB_G2(true, true, ACCUM) TB_G2(true, true, MEM_UPDATE) TB_G2(true, true, PARTIAL)
  TB_G2(true, false, STORE) TB_G2(true, false, PARTIAL)
#undef TB_G2
  TORCH_CHECK(false, "gemm_sm100: no kernel for this layout / epilogue");
launched:
  check_launch("gemm_sm100");
  if (kmode == PARTIAL) {
    const int64_t total = (int64_t)a.tiles * HM * CG * (BN / 8);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((total + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, (const float*)ws.data_ptr<float>(), a));
    check_launch("gemm_sm100 split-K reduce");
  }
}

}  // namespace tb
