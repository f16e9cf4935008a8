"""Data-parallel engine: one process per GPU, replicated model, averaged gradients.

The reference gets data parallelism from Accelerate -> torch DDP
(`scripts/pretrain_distributed.py:350-413`): bucketed fp32 all-reduce from
autograd hooks, with ``find_unused_parameters=False`` (which raises at the
second iteration because the memory gates and key/value projections never
receive gradients).  Here the gradients live in the optimizer's flat buffer,
parameters that got no gradient are simply left out of the update, and the
reduction runs over that buffer:

* ``reduce="nccl"``: one NCCL all-reduce of the flat gradient (the baseline
  path; bf16 on the wire, averaged by the optimizer's gradient scale).
* ``reduce="fused"``: the peer-memory kernel in ``csrc/comm.cu`` that
  reduce-scatters the flat gradient over NVLink, applies clip + AdamW to the
  local shard and all-gathers the new weights in one launch (see
  :mod:`titans_pytorch_b200.parallel.fused`).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..train.optim import FusedAdamW


class DPFusedAdamW(FusedAdamW):
    def __init__(self, *a, world_size: int = 1, **kw):
        super().__init__(*a, **kw)
        self.world_size = world_size

    def grad_scale(self) -> float:
        return 1.0 / self.world_size


class DataParallelEngine:
    def __init__(self, group=None, reduce: str = "nccl") -> None:
        if not dist.is_initialized():
            raise RuntimeError("DataParallelEngine needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.reduce = reduce

    def make_optimizer(self, model: torch.nn.Module, cfg) -> DPFusedAdamW:
        opt = DPFusedAdamW(model.parameters(), lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                           weight_decay=cfg.weight_decay, max_grad_norm=cfg.grad_clip,
                           world_size=self.world,
                           use_kernels=getattr(getattr(model, "config", None), "use_kernels", None))
        # identical starting weights on every rank
        dist.broadcast(opt.space.flat, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                       group=self.group)
        if opt.master is not opt.space.flat:
            opt.master.copy_(opt.space.flat)
        self._sync_buffers(model)
        return opt

    def _sync_buffers(self, model):
        for b in model.buffers():
            dist.broadcast(b, src=0, group=self.group)

    def reduce_gradients(self, optimizer: DPFusedAdamW) -> None:
        """Sum the flat gradient over ranks (the optimizer divides by world size)."""
        # Ranks must agree on which parameters received gradients.  The set is a
        # property of the model structure, so it is agreed once (a small
        # all-reduce + host read) and reused while the local set is unchanged.
        local = tuple(optimizer.space.got)
        if local != getattr(self, "_last_local", None):
            got = torch.tensor(local, dtype=torch.uint8, device=optimizer.space.device)
            dist.all_reduce(got, op=dist.ReduceOp.MAX, group=self.group)
            self._last_local = local
            self._agreed = [bool(x) for x in got.tolist()]
        optimizer.space.got = list(self._agreed)
        dist.all_reduce(optimizer.space.grad, group=self.group)
