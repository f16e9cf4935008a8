"""Context parallelism for MAG / MAL / LMM: the sequence split across ranks.

The reference has no sequence or context parallelism; it reaches long contexts
by the MAC chunk recurrence, sliding-window attention and cross-call state
carry (`src/titans/models.py:301-314`, `src/titans/attention.py:135-307`).
This module shards one sequence of ``S`` tokens into ``world`` contiguous
pieces of ``T = S / world`` tokens, one per rank, and keeps the result equal to
the unsharded model:

* Sliding-window attention needs, for a query at global token ``g``, the keys
  ``g - w + 1 .. g``: a halo of the previous rank's last ``w - 1`` rows.
  :func:`halo_exchange` sends those rows forward over one point-to-point
  exchange (NCCL over NVLink on GPUs, gloo on CPU) and, in the backward, sends
  their gradient back to the rank that owns them.  RoPE positions are global
  (``window_attention(..., pos_offset)``).
* The memory's causal depthwise convolutions need ``K - 1`` halo rows.
* In ``ref`` semantics the memory update reads the whole sequence only through
  two sums: the mean of the memory input that drives the gates
  (`src/titans/memory.py:427-431`) and the associative-loss gradient, a sum of
  per-token outer products scaled by ``2 / (B * S * D)``
  (`src/titans/memory.py:287-349`, `:180`).  Both are the average of the per-shard
  values over the ranks, so one all-reduce each makes every rank's new state
  the unsharded one.  Retrieval uses the incoming state only, so nothing else
  in the memory crosses ranks.

Parameters stay replicated: run the step under a data-parallel engine on the
same process group so their gradients are averaged, which equals the
gradient of the whole sequence's mean loss (every shard has ``T`` tokens).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ContextShard:
    """This rank's place in a context-parallel group."""

    group: object = None
    rank: int = 0
    world: int = 1

    @classmethod
    def from_group(cls, group=None) -> "ContextShard":
        if not dist.is_available() or not dist.is_initialized():
            return cls(None, 0, 1)
        return cls(group, dist.get_rank(group), dist.get_world_size(group))

    @property
    def active(self) -> bool:
        return self.world > 1

    def _global(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def extend(self, x: torch.Tensor, rows: int) -> tuple[torch.Tensor, int]:
        """``[prev rank's last rows || x]`` and the number of rows prepended."""
        if not self.active or rows <= 0:
            return x, 0
        if rows > x.shape[1]:
            raise ValueError(f"a halo of {rows} rows needs shards of at least that many tokens "
                             f"(got {x.shape[1]})")
        return halo_exchange(x, rows, self), (rows if self.rank > 0 else 0)

    def start(self, local_len: int) -> int:
        """Global index of this rank's first token (every shard has ``local_len``)."""
        return self.rank * local_len

    def all_reduce_mean_(self, t: torch.Tensor) -> torch.Tensor:
        if self.active:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            t.div_(self.world)
        return t


def _exchange(send: torch.Tensor | None, recv: torch.Tensor | None, to: int | None, frm: int | None, group):
    ops = []
    if send is not None:
        ops.append(dist.P2POp(dist.isend, send.contiguous(), to, group))
    if recv is not None:
        ops.append(dist.P2POp(dist.irecv, recv, frm, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class _HaloExchange(torch.autograd.Function):
    """Forward: rank r receives rank r-1's last ``rows`` rows and prepends them.
    Backward: the gradient of those rows returns to rank r-1 and adds into the
    gradient of its last rows."""

    @staticmethod
    def forward(ctx, x, rows, shard):
        r, w = shard.rank, shard.world
        nxt = shard._global(r + 1) if r + 1 < w else None
        prv = shard._global(r - 1) if r > 0 else None
        B, _, D = x.shape
        halo = torch.empty(B, rows, D, dtype=x.dtype, device=x.device) if prv is not None else None
        _exchange(x[:, -rows:] if nxt is not None else None, halo, nxt, prv, shard.group)
        ctx.rows, ctx.shard, ctx.nxt, ctx.prv = rows, shard, nxt, prv
        if halo is None:
            return x.view_as(x)
        return torch.cat([halo, x], dim=1)

    @staticmethod
    def backward(ctx, dy):
        rows = ctx.rows
        dy = dy.contiguous()
        if ctx.prv is not None:
            dhalo, dx = dy[:, :rows], dy[:, rows:].clone()
        else:
            dhalo, dx = None, dy.clone()
        dtail = torch.empty_like(dx[:, -rows:]) if ctx.nxt is not None else None
        _exchange(dhalo, dtail, ctx.prv, ctx.nxt, ctx.shard.group)
        if dtail is not None:
            dx[:, -rows:] += dtail
        return dx, None, None


def halo_exchange(x: torch.Tensor, rows: int, shard: ContextShard) -> torch.Tensor:
    """``x`` [B, T, D] -> ``[halo || x]`` with the previous rank's last ``rows``
    rows (rank 0 gets ``x`` back).  Every rank of the group must call it."""
    return _HaloExchange.apply(x, int(rows), shard)


def shard_sequence(t: torch.Tensor, shard: ContextShard, dim: int = 1) -> torch.Tensor:
    """This rank's contiguous piece of a ``[B, S, ...]`` tensor."""
    S = t.shape[dim]
    if S % shard.world:
        raise ValueError(f"sequence length {S} is not divisible by the context-parallel size {shard.world}")
    T = S // shard.world
    return t.narrow(dim, shard.rank * T, T)


def shard_batch(batch: dict, shard: ContextShard) -> dict:
    """``input_ids`` / ``labels`` (already shifted over the whole sequence) of this rank."""
    return {k: (shard_sequence(v, shard) if torch.is_tensor(v) and v.dim() >= 2 else v)
            for k, v in batch.items()}


class ShardedLoader:
    """Wrap a loader that yields the same whole-sequence batches on every rank
    so that each rank receives its own sequence shard of them."""

    def __init__(self, loader, shard: ContextShard) -> None:
        self.loader, self.shard = loader, shard

    def __iter__(self):
        for b in self.loader:
            yield shard_batch(b, self.shard)

    def __len__(self) -> int:
        return len(self.loader)


def enable_context_parallel(model, group=None) -> ContextShard:
    """Put a MAG / MAL / LMM model into context-parallel mode on ``group``.

    Every block exchanges halos with its neighbours and every memory update
    averages its statistics over the group.  ``ref`` semantics only: the paper
    mode's per-token scan is a recurrence over the whole sequence.
    """
    mt = getattr(model, "model_type", None)
    if mt not in ("mag", "mal", "lmm"):
        raise NotImplementedError(f"context parallelism covers MAG, MAL and LMM, not {mt!r}: MAC's "
                                  "chunk recurrence is sequential over the sequence")
    if model.config.semantics != "ref":
        raise NotImplementedError("context parallelism needs semantics='ref'")
    shard = ContextShard.from_group(group)
    for block in model.blocks:
        block.cp = shard
        block.memory.cp = shard
    return shard


def disable_context_parallel(model) -> None:
    for block in model.blocks:
        block.cp = None
        block.memory.cp = None


__all__ = ["ContextShard", "ShardedLoader", "halo_exchange", "shard_sequence", "shard_batch",
           "enable_context_parallel", "disable_context_parallel"]
