"""tcgen05 GEMM and the fused all-gather + GEMM of sharded parameters.

``gemm(a, b)`` is ``a @ b.T`` on the persistent sm_100a kernel in
``csrc/gemm_tc.cu`` (bf16 operands, fp32 accumulation).  Plain GEMMs in the
models stay on cuBLAS; this kernel exists for the fused form:

``gemm_gather(a, b, flat, src_ptrs, u0, length, shard, rank, consume)``
computes ``a @ b.T`` while it all-gathers flat elements ``[u0, u0 + length)``
of this rank's parameter buffer from the ranks that own them (rank ``r`` owns
unit-relative ``[r * shard, (r + 1) * shard)``; ``src_ptrs`` holds every
rank's buffer address, peer pointers included).  With ``consume`` the weight
``b`` is a view of ``flat`` inside the unit and each output tile waits for its
weight rows; otherwise ``b`` is already local and the gather is a prefetch
that runs under the tensor-core tiles.  ``gather(flat, ...)`` is the same
all-gather as a standalone kernel.
"""

from __future__ import annotations

import torch

from ._ext import ext


def gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M, K] @ b [N, K].T`` (bf16, K and N multiples of 8)."""
    return ext().gemm_tc(a.contiguous(), b.contiguous())


def gemm_gather(a: torch.Tensor, b: torch.Tensor, flat: torch.Tensor, src_ptrs: torch.Tensor, u0: int,
                length: int, shard: int, rank: int, consume: bool) -> torch.Tensor:
    return ext().gemm_gather_tc(a, b, flat, src_ptrs, int(u0), int(length), int(shard), int(rank), bool(consume))


def gather(flat: torch.Tensor, src_ptrs: torch.Tensor, u0: int, length: int, shard: int, rank: int) -> None:
    ext().fsdp_gather(flat, src_ptrs, int(u0), int(length), int(shard), int(rank))


__all__ = ["gemm", "gemm_gather", "gather"]
