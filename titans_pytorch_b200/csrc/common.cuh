// Shared device helpers for the titans_pytorch_b200 kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "device_common.cuh"

#define TB_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define TB_CHECK_LASTDIM(x) TORCH_CHECK((x).stride(-1) == 1, #x " must have a contiguous last dim")

namespace tb {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

inline int num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

inline bool aligned16(const at::Tensor& t) { return ((uintptr_t)t.data_ptr() % 16) == 0; }

// Contiguous and 16-byte aligned view of t (copies only when needed), so
// 16-byte vector loads/stores in the kernels are always legal.
inline at::Tensor contig16(const at::Tensor& t) {
  at::Tensor c = t.contiguous();
  if (!aligned16(c)) c = c.clone(at::MemoryFormat::Contiguous);
  return c;
}

inline void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

inline int act_code(const std::string& s) {
  if (s == "silu") return ACT_SILU;
  if (s == "gelu") return ACT_GELU;
  if (s == "relu") return ACT_RELU;
  if (s == "none") return ACT_NONE;
  TORCH_CHECK(false, "unknown activation ", s);
}

}  // namespace tb

// Dispatch over the floating types the kernels support.
#define TB_DISPATCH_FLOAT(dtype, NAME, ...)                                   \
  [&] {                                                                       \
    if ((dtype) == at::kBFloat16) {                                           \
      using scalar_t = __nv_bfloat16;                                         \
      return __VA_ARGS__();                                                   \
    } else if ((dtype) == at::kFloat) {                                       \
      using scalar_t = float;                                                 \
      return __VA_ARGS__();                                                   \
    } else if ((dtype) == at::kHalf) {                                        \
      using scalar_t = __half;                                                \
      return __VA_ARGS__();                                                   \
    }                                                                         \
    TORCH_CHECK(false, NAME, ": unsupported dtype ", dtype);                  \
  }()
