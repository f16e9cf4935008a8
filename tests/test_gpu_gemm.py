"""tcgen05 GEMM and fused all-gather + GEMM vs fp32 PyTorch.

The gather runs over ranks emulated on one GPU: every "rank" is a separate
buffer of this device holding the current values of its own shard only; the
kernel sees them through the same pointer table it gets from peer GPUs.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs CUDA", allow_module_level=True)

from titans_pytorch_b200.ops import _ext  # noqa: E402
from titans_pytorch_b200.ops.gemm import gather, gemm, gemm_gather  # noqa: E402

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _status():
    return int(_ext.ext().kernel_error_status(0, True))


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (300, 264, 200), (128, 256, 64), (2048, 2304, 768),
                                   (4100, 1024, 1536), (77, 8, 24)])
def test_gemm_tc(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    b = torch.randn(N, K, device=DEV, dtype=torch.bfloat16)
    c = gemm(a, b)
    torch.cuda.synchronize()
    assert _status() == 0
    ref = a.float() @ b.float().t()
    assert c.shape == (M, N) and c.dtype == torch.bfloat16
    assert rel_err(c, ref) < 1e-2


def _emulated_ranks(world, total, u0, length, seed=0):
    """Truth buffer plus one buffer per rank whose unit holds only its own shard
    (the rest is garbage), and the shard size."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    truth = torch.randn(total, device=DEV, dtype=torch.bfloat16, generator=g)
    shard = -(-length // world // 8) * 8
    bufs = []
    for r in range(world):
        b = torch.full((total,), float("nan"), device=DEV, dtype=torch.bfloat16)
        b[:u0] = truth[:u0]
        b[u0 + length:] = truth[u0 + length:]
        lo, hi = u0 + r * shard, min(u0 + (r + 1) * shard, u0 + length)
        if hi > lo:
            b[lo:hi] = truth[lo:hi]
        bufs.append(b)
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=DEV)
    return truth, bufs, ptrs, shard


@pytest.mark.parametrize("world,me", [(3, 1), (8, 5), (2, 0)])
@pytest.mark.parametrize("M,N,K", [(200, 264, 96), (1024, 768, 256)])
def test_gemm_gather_consume(world, me, M, N, K):
    torch.manual_seed(1)
    u0, pre, post = 4096, 1000 * 8, 333 * 8
    length = pre + N * K + post
    total = u0 + length + 512
    truth, bufs, ptrs, shard = _emulated_ranks(world, total, u0, length)
    w0 = u0 + pre
    flat = bufs[me]
    w = flat[w0:w0 + N * K].view(N, K)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    c = gemm_gather(a, w, flat, ptrs, u0, length, shard, me, consume=True)
    torch.cuda.synchronize()
    assert _status() == 0
    assert torch.equal(flat, truth), "the unit must be fully gathered"
    ref = a.float() @ truth[w0:w0 + N * K].view(N, K).float().t()
    assert rel_err(c, ref) < 1e-2


@pytest.mark.parametrize("world,me", [(4, 2), (8, 0)])
def test_gemm_gather_prefetch(world, me):
    torch.manual_seed(2)
    u0, length = 8192, 3 * 1000 * 1000 + 8 * 77
    total = u0 + length + 64
    truth, bufs, ptrs, shard = _emulated_ranks(world, total, u0, length, seed=3)
    a = torch.randn(513, 512, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(384, 512, device=DEV, dtype=torch.bfloat16)
    c = gemm_gather(a, w, bufs[me], ptrs, u0, length, shard, me, consume=False)
    torch.cuda.synchronize()
    assert _status() == 0
    assert torch.equal(bufs[me], truth)
    assert rel_err(c, a.float() @ w.float().t()) < 1e-2


def test_plain_gather():
    world, me = 5, 3
    u0, length = 800, 123456 * 8
    total = u0 + length + 8
    truth, bufs, ptrs, shard = _emulated_ranks(world, total, u0, length, seed=4)
    gather(bufs[me], ptrs, u0, length, shard, me)
    torch.cuda.synchronize()
    assert torch.equal(bufs[me], truth)
