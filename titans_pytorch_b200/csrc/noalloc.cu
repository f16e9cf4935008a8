// Allocation-free RMSNorm backward (see noalloc.h for the contract).
//
// No counterpart in the reference.  Callers that cannot allocate GPU memory
// (allocator/OOM-handler code, non-PyTorch hosts that only lend their own
// buffers, loops that forbid synchronising cudaMalloc/cudaFree) get the same
// kernels as the PyTorch entry point, with the dweight partial sums placed in
// a file-scope device array instead of a per-call allocation.
#include <algorithm>
#include <mutex>

#include "noalloc.h"
#include "norm_kernels.cuh"

namespace {

constexpr int kScratchFloats = TITANS_NOALLOC_RMS_SCRATCH_FLOATS;
constexpr int kMaxDevices = 64;

// Scratch for the per-block dweight partials (rows of `dim` floats).  In host
// code this name is only a stand-in for the symbol: its device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_rms_bwd_scratch[kScratchFloats];

float* g_scratch_ptr[kMaxDevices];  // device address per device, set once
int g_num_sms[kMaxDevices];
std::mutex g_setup_mutex;

// Once per device, with that device current: resolve the scratch address.
// The address and SM count are handed back while the lock is held, so no
// caller reads the per-device tables unsynchronised.
int setup_device(int dev, float** scratch, int* nsm) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] != nullptr) {
    *scratch = g_scratch_ptr[dev];
    *nsm = g_num_sms[dev];
    return TITANS_NOALLOC_OK;
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_rms_bwd_scratch) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return TITANS_NOALLOC_ESETUP;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return TITANS_NOALLOC_ESETUP;
  }
  g_num_sms[dev] = n;
  g_scratch_ptr[dev] = static_cast<float*>(p);
  *scratch = g_scratch_ptr[dev];
  *nsm = n;
  return TITANS_NOALLOC_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <typename T, int CH>
int launch(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw, int64_t rows,
           int dim, int blocks, float* scratch, cudaStream_t st) {
  const int threads = 256;
  const size_t smem = (size_t)(threads / 32) * dim * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(tb::rms_bwd_kernel<T, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess) {
    cudaGetLastError();
    return TITANS_NOALLOC_ELAUNCH;
  }
  tb::rms_bwd_kernel<T, CH><<<blocks, threads, smem, st>>>(
      static_cast<const T*>(dy), static_cast<const T*>(x), static_cast<const T*>(w), rstd, static_cast<T*>(dx),
      scratch, rows, dim);
  tb::colsum_kernel<<<(dim + 255) / 256, 256, 0, st>>>(scratch, dw, blocks, dim);
  return cudaGetLastError() == cudaSuccess ? TITANS_NOALLOC_OK : TITANS_NOALLOC_ELAUNCH;
}

template <typename T>
int dispatch(int chn, const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
             int64_t rows, int dim, int blocks, float* scratch, cudaStream_t st) {
  switch (chn) {
    case 1: return launch<T, 1>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    case 2: return launch<T, 2>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    case 3: return launch<T, 3>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    case 4: return launch<T, 4>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    case 5: case 6: return launch<T, 6>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    case 7: case 8: return launch<T, 8>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
    default: return launch<T, 16>(dy, x, w, rstd, dx, dw, rows, dim, blocks, scratch, st);
  }
}

}  // namespace

extern "C" int titans_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* weight, const float* rstd,
                                           void* dx, float* dweight, int64_t rows, int32_t dim, int32_t dtype,
                                           void* stream) {
  if (dtype != TITANS_DTYPE_F32 && dtype != TITANS_DTYPE_BF16) return TITANS_NOALLOC_EINVAL;
  const int V = dtype == TITANS_DTYPE_BF16 ? 8 : 4;  // elements per 16-byte vector
  if (rows < 0 || dim <= 0 || dim % V != 0) return TITANS_NOALLOC_EINVAL;
  const int chn = (dim + 32 * V - 1) / (32 * V);
  if (chn > 16 || dim > kScratchFloats) return TITANS_NOALLOC_ETOOBIG;
  if (dweight == nullptr || weight == nullptr || !aligned(weight, 16) || !aligned(dweight, 4))
    return TITANS_NOALLOC_EINVAL;
  if (rows > 0 && (dy == nullptr || x == nullptr || dx == nullptr || rstd == nullptr || !aligned(dy, 16) ||
                   !aligned(x, 16) || !aligned(dx, 16) || !aligned(rstd, 4)))
    return TITANS_NOALLOC_EINVAL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return TITANS_NOALLOC_EINVAL;
  }
  float* scratch = nullptr;
  int nsm = 0;
  const int rc = setup_device(dev, &scratch, &nsm);
  if (rc != TITANS_NOALLOC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    return cudaMemsetAsync(dweight, 0, (size_t)dim * sizeof(float), st) == cudaSuccess ? TITANS_NOALLOC_OK
                                                                                       : TITANS_NOALLOC_ELAUNCH;
  }
  // same block count as the PyTorch entry point, capped so the partials fit the scratch array
  int64_t blocks = std::min<int64_t>((rows + 7) / 8, (int64_t)nsm * 2);
  blocks = std::max<int64_t>(1, std::min<int64_t>(blocks, kScratchFloats / dim));
  if (dtype == TITANS_DTYPE_BF16)
    return dispatch<__nv_bfloat16>(chn, dy, x, weight, rstd, dx, dweight, rows, dim, (int)blocks, scratch, st);
  return dispatch<float>(chn, dy, x, weight, rstd, dx, dweight, rows, dim, (int)blocks, scratch, st);
}

extern "C" const char* titans_noalloc_strerror(int code) {
  switch (code) {
    case TITANS_NOALLOC_OK: return "ok";
    case TITANS_NOALLOC_EINVAL:
      return "invalid argument: null or misaligned pointer, unknown dtype, or dim not a multiple of the 16-byte "
             "vector width";
    case TITANS_NOALLOC_ETOOBIG:
      return "size beyond the maximum: dim must be at most 4096 (bf16) / 2048 (fp32) and fit the 4 MiB scratch array";
    case TITANS_NOALLOC_ESETUP: return "could not resolve the device address of the static scratch array";
    case TITANS_NOALLOC_ELAUNCH: return "kernel launch failed";
    default: return "unknown error code";
  }
}
