"""The allocation-free C entry point ``titans_rms_norm_bwd_noalloc``.

Some callers cannot allocate GPU memory when they call into the library (an
allocator or out-of-memory handler, a host runtime that only lends its own
buffers, a loop that must not synchronise on cudaMalloc/cudaFree).  They call
this exported C symbol with their own input and output buffers; its scratch
space is a fixed device array inside the library.  These tests call it through
ctypes and compare it with the library's PyTorch-facing ``rms_norm_bwd`` on two
calls in a row (the shared scratch array must not leak state between calls).
Each call is also checked against an fp32 PyTorch restatement of the RMSNorm
backward, so the test does not rest on the other entry point alone.
This file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs CUDA", allow_module_level=True)

from titans_pytorch_b200.ops import _ext  # noqa: E402

OK, EINVAL, ETOOBIG = 0, 1, 2
DTYPES = {torch.float32: 0, torch.bfloat16: 1}


def _lib():
    lib = ctypes.CDLL(_ext.so_path())
    fn = lib.titans_rms_norm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
    err = lib.titans_noalloc_strerror
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, dy, x, w, rstd, dx, dw):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(),
              x.shape[0], x.shape[1], DTYPES[x.dtype], stream)


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def rms_bwd_fp32(dy, x, w, eps=1e-6):
    """fp32 restatement: y = x * r * w with r = (mean(x^2) + eps)^-1/2."""
    x, dy, w = x.float(), dy.float(), w.float()
    r = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    xh = x * r
    g = dy * w
    dx = r * (g - xh * (g * xh).mean(-1, keepdim=True))
    dw = (dy * xh).sum(0)
    return dx, dw


@pytest.mark.parametrize("dtype,rows,dim", [(torch.bfloat16, 4096, 768), (torch.bfloat16, 37, 1536),
                                             (torch.float32, 300, 1024), (torch.bfloat16, 5, 4096)])
def test_noalloc_matches_torch_entry_point_twice(dtype, rows, dim):
    fn, _ = _lib()
    E = _ext.ext()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    for call in range(2):  # two calls in a row through the shared scratch array
        torch.manual_seed(100 + call)
        x = torch.randn(rows, dim, device="cuda", dtype=dtype)
        w = (1 + 0.1 * torch.randn(dim, device="cuda")).to(dtype)
        dy = torch.randn(rows, dim, device="cuda", dtype=dtype)
        _, rstd = E.rms_norm_fwd(x, w, 1e-6)
        dx_ref, dw_ref = E.rms_norm_bwd(dy, x, w, rstd, True)
        dx = torch.empty_like(x)
        dw = torch.full((dim,), float("nan"), device="cuda", dtype=torch.float32)
        rc = _call(fn, dy, x, w, rstd, dx, dw)
        torch.cuda.synchronize()
        assert rc == OK
        assert rel_err(dx, dx_ref) < tol
        assert rel_err(dw, dw_ref) < tol
        dx32, dw32 = rms_bwd_fp32(dy, x, w)
        assert rel_err(dx, dx32) < tol
        assert rel_err(dw, dw32) < tol


def test_noalloc_rejects_sizes_beyond_the_maximum():
    fn, err = _lib()
    dim = 8192  # beyond the bf16 limit of 4096
    x = torch.zeros(8, dim, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(dim, device="cuda", dtype=torch.bfloat16)
    rstd = torch.ones(8, device="cuda")
    dx = torch.empty_like(x)
    dw = torch.empty(dim, device="cuda")
    rc = _call(fn, x, x, w, rstd, dx, dw)
    assert rc == ETOOBIG
    assert b"maximum" in err(rc)
    x2 = torch.zeros(8, 100, device="cuda", dtype=torch.bfloat16)  # not a multiple of 8 bf16 values
    w2 = torch.ones(100, device="cuda", dtype=torch.bfloat16)
    rc2 = _call(fn, x2, x2, w2, rstd, torch.empty_like(x2), torch.empty(100, device="cuda"))
    assert rc2 == EINVAL
