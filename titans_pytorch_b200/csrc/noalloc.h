/* Allocation-free C entry point of the kernel library.
 *
 * This interface has no counterpart in the reference (Aedelon/titans-pytorch
 * has no native code at all).  It exists for callers that cannot allocate GPU
 * memory at the time they call: code running inside a custom allocator or an
 * out-of-memory handler, host runtimes that hand the library only the buffers
 * they own (a C/C++ or foreign-language host without PyTorch's caching
 * allocator), and hot loops whose owners forbid cudaMalloc/cudaFree because
 * they synchronise the device.  Such a caller passes its own input and output
 * buffers; the scratch space the kernel needs lives in a fixed-size
 * device-global array inside the library instead of being allocated per call.
 *
 * titans_rms_norm_bwd_noalloc
 *   The RMSNorm backward pass (same kernels and results as the library's
 *   PyTorch-facing rms_norm_bwd):
 *     dx      = rstd * (dy*w - xhat * mean(dy*w*xhat)),  xhat = x * rstd
 *     dweight = sum over rows of dy * xhat   (fp32)
 *   Arguments are device pointers: dy, x, dx are [rows, dim] row-major of the
 *   given dtype; weight is [dim] of the same dtype; rstd is [rows] fp32 (the
 *   reciprocal RMS saved by the forward); dweight is [dim] fp32.  dy, x, dx and
 *   weight must be 16-byte aligned.  `stream` is a cudaStream_t (NULL = legacy
 *   default stream).  The call is asynchronous on that stream.
 *
 *   Scratch: the per-block partial sums of dweight go to a static device array
 *   of TITANS_NOALLOC_RMS_SCRATCH_FLOATS floats (4 MiB) that every GPU loading
 *   the library holds until the process exits.  The number of blocks is capped
 *   so the partials fit; dim larger than the kernel's limit (4096 for bf16,
 *   2048 for fp32) is rejected with TITANS_NOALLOC_ETOOBIG.  Every call
 *   rewrites the part of the array it reads, so no state carries over between
 *   calls, but all calls on a device share the one array: calls that can
 *   overlap on the GPU (different streams without ordering between them) race
 *   and must not be issued.
 *
 *   Set-up: the first call on each device (with that device current) looks up
 *   the array's device address with cudaGetSymbolAddress and caches it; make
 *   that first call before any stream capture.  No call allocates memory.
 *
 *   Returns TITANS_NOALLOC_OK or an error code; titans_noalloc_strerror gives
 *   a message for it.
 */
#ifndef TITANS_NOALLOC_H
#define TITANS_NOALLOC_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TITANS_NOALLOC_OK = 0,
  TITANS_NOALLOC_EINVAL = 1,   /* null/misaligned pointer, bad dtype, dim not a multiple of the vector width */
  TITANS_NOALLOC_ETOOBIG = 2,  /* dim beyond the kernel's limit or the scratch array's size */
  TITANS_NOALLOC_ESETUP = 3,   /* the scratch array's device address could not be obtained */
  TITANS_NOALLOC_ELAUNCH = 4   /* a kernel launch failed */
};

enum { TITANS_DTYPE_F32 = 0, TITANS_DTYPE_BF16 = 1 };

#define TITANS_NOALLOC_RMS_SCRATCH_FLOATS (1 << 20)

int titans_rms_norm_bwd_noalloc(const void* dy, const void* x, const void* weight, const float* rstd, void* dx,
                                float* dweight, int64_t rows, int32_t dim, int32_t dtype, void* stream);

const char* titans_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif

#endif /* TITANS_NOALLOC_H */
