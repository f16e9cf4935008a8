"""Data-parallel engine: one process per GPU, replicated model, averaged gradients.

The reference gets data parallelism from Accelerate -> torch DDP
(`scripts/pretrain_distributed.py:350-413`): bucketed fp32 all-reduce from
autograd hooks, with ``find_unused_parameters=False``, which raises at the
second iteration because the memory gates and key/value projections never
receive gradients.  Here gradients live in the optimizer's flat buffer,
parameters that got no gradient this step are left out of the update (the
ranks agree on that set once), and the reduction runs over the flat buffer:

* ``reduce="fused"`` (default on CUDA): ``csrc/comm.cu``.  The flat bf16
  gradient and parameter buffers are peer-visible (CUDA IPC over NVLink).
  Each rank reduce-scatters its shard by loading the peers' gradients
  directly, the shard norms are exchanged through peer slots for the global
  clip, and one kernel applies AdamW to the shard and stores the new bf16
  weights into every rank's parameter buffer (all-gather by peer stores).
  Optimizer state (fp32 master, moments) exists only for the local shard
  (ZeRO-1).  All cross-GPU waits are bounded flag barriers.
* ``reduce="collective"``: one ``torch.distributed.all_reduce`` of the flat
  gradient (NCCL on GPUs, gloo on CPU), then the replicated fused AdamW.  This
  is the library-collective baseline and the path CPU tests use.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext
from .peer import PeerBuffer
from ..train.optim import (ALIGN, FlatParamSpace, FusedAdamW, intersect_segments, segment_table,
                           unique_trainable)


class DPFusedAdamW(FusedAdamW):
    """Replicated AdamW over an all-reduced flat gradient (collective path)."""

    def __init__(self, *a, world_size: int = 1, **kw):
        super().__init__(*a, **kw)
        self.world_size = world_size

    def grad_scale(self) -> float:
        return 1.0 / self.world_size


_PeerBuffer = PeerBuffer  # kept for callers of the former name


class FusedDPAdamW(FusedAdamW):
    """ZeRO-1 AdamW whose step is the fused peer-memory reduce + update + all-gather."""

    # each rank holds only its shard of the optimizer state: checkpoints keep one file per rank
    shard_state = True

    def __init__(self, model: torch.nn.Module, cfg, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        params = unique_trainable(model.parameters())
        device = params[0].device if device is None else device
        if params[0].dtype != torch.bfloat16:
            raise ValueError("the fused data-parallel path runs bf16 parameters")
        self._bufs = []

        def peer_buffers(total, dtype):
            nbytes = total * 2
            fb = _PeerBuffer(nbytes, device, group, self.world, self.rank)
            gb = _PeerBuffer(nbytes, device, group, self.world, self.rank)
            self._bufs += [fb, gb]
            self._param_buf, self._grad_buf = fb, gb
            return fb.local.view(torch.bfloat16), gb.local.view(torch.bfloat16)

        space = FlatParamSpace(params, pad_to=ALIGN * self.world, buffers=peer_buffers)
        self.sig = _PeerBuffer(4 * 4 * self.world, device, group, self.world, self.rank)
        self.slots = _PeerBuffer(4 * self.world, device, group, self.world, self.rank)
        self._bufs += [self.sig, self.slots]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast(space.flat, src=src, group=group)
        for b in model.buffers():
            dist.broadcast(b, src=src, group=group)
        torch.optim.Optimizer.__init__(self, space.params, dict(lr=cfg.lr, betas=tuple(cfg.betas), eps=cfg.eps,
                                                                 weight_decay=cfg.weight_decay))
        self.space = space
        self.max_grad_norm = float(cfg.grad_clip)
        self.kernels = True
        self.n = space.total // self.world
        self.lo = self.rank * self.n
        self.master = space.flat[self.lo:self.lo + self.n].float()
        self.exp_avg = torch.zeros(self.n, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(self.n, dtype=torch.float32, device=device)
        self.gsum = torch.empty(self.n, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.norm_out = torch.zeros(1, dtype=torch.float32, device=device)
        self.last_grad_norm = self.norm_out
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)  # advanced by the first barrier
        self.step_count = 0
        self._tab_key = None
        self.graph_safe = True

    def grad_scale(self) -> float:
        return 1.0 / self.world

    def _shard_table(self):
        segs = self.space.active_segments()
        key = tuple(segs)
        if key != self._tab_key:
            self._tab = segment_table(intersect_segments(segs, self.lo, self.lo + self.n), self.space.device)
            self._tab_key = key
        return self._tab

    @torch.no_grad()
    def step(self, closure=None, hyper: torch.Tensor | None = None, schedule: tuple | None = None):
        """One fused step; ``hyper``/``schedule`` as in :meth:`FusedAdamW.step`
        (device-side step count and learning rate for CUDA-graph replay)."""
        loss = closure() if closure is not None else None
        E = ext()
        g = self.param_groups[0]
        self.step_count += 1
        tab, nseg, items = self._shard_table()
        w, me = self.world, self.rank
        lr, b1, b2 = g["lr"], g["betas"][0], g["betas"][1]
        if hyper is not None:
            warm, total, mr = schedule if schedule is not None else (0, 1, 1.0)
            E.adamw_hyper_step(hyper, g.get("initial_lr", lr), b1, b2, warm, total, mr, schedule is not None)
        E.comm_barrier(self.sig.ptrs, 0, self.epoch, True, w, me, self.err)   # all gradients complete
        E.comm_reduce_shard(self._grad_buf.ptrs, self.lo, self.n, self.gsum, self.grad_scale(),
                            self.slots.ptrs, w, me)
        E.comm_barrier(self.sig.ptrs, 1, self.epoch, False, w, me, self.err)  # all shard norms published
        E.comm_adamw_shard(self.gsum, self.master, self.exp_avg, self.exp_avg_sq, self._param_buf.ptrs,
                           self.lo, w, tab, nseg, items, self.slots.local.view(torch.float32),
                           self.grad_scale(), self.max_grad_norm, lr, b1, b2, g["eps"], g["weight_decay"],
                           self.step_count, self.norm_out, hyper)
        E.comm_barrier(self.sig.ptrs, 2, self.epoch, False, w, me, self.err)  # every rank's weights written
        return loss

    def comm_bytes(self) -> int:
        """Device bytes held outside PyTorch's allocator (the peer-visible buffers)."""
        return sum(b.nbytes for b in self._bufs)

    def check_errors(self) -> None:
        """Raise if a bounded cross-GPU wait ran out (reads a device word: synchronises)."""
        v = int(self.err.item())
        if v:
            raise RuntimeError(f"fused data-parallel step: cross-GPU wait timed out (code {v})")

    def state_dict(self):
        return {"step": self.step_count, "shard": (self.lo, self.n), "master": self.master,
                "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq,
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, sd):
        if tuple(sd["shard"]) != (self.lo, self.n):
            raise ValueError("optimizer shard layout differs (world size changed?)")
        self.step_count = int(sd["step"])
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for pg, sg in zip(self.param_groups, sd["param_groups"]):
            pg.update(sg)

    def close(self):
        for b in self._bufs:
            b.close()


class DataParallelEngine:
    """Engine for :class:`~titans_pytorch_b200.train.trainer.Trainer` (``engine=``).

    ``reduce="fused"`` (default on CUDA): one contiguous optimizer shard per
    rank; after the backward one fused peer-memory reduce-scatter, clip, AdamW
    on the shard and the all-gather by peer stores (:class:`FusedDPAdamW`).
    ``overlap=True``: the optimizer state is sharded per block
    (:class:`~titans_pytorch_b200.parallel.fsdp.FSDPAdamW` with every unit
    replicated) and each block's gradients are reduce-scattered on a
    communication stream as soon as the backward has finished with the block
    (DDP's bucketed all-reduce from autograd hooks).  Measured on the TitansMAG
    ~170M step at 8 GPUs, the post-backward exchange costs about 1.6 ms of a
    75 ms step (mostly the AdamW shard and the all-gather, which overlap does
    not hide) and the per-block barriers and reduce CTAs beside the backward's
    GEMMs cost more than they hide (76.1 vs 74.9 ms), so it is off by default."""

    def __init__(self, group=None, reduce: str | None = None, overlap: bool = False) -> None:
        if not dist.is_initialized():
            raise RuntimeError("DataParallelEngine needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if reduce is None:
            reduce = "fused" if (torch.cuda.is_available() and dist.get_backend(group) == "nccl") else "collective"
        if reduce not in ("fused", "collective"):
            raise ValueError("reduce must be 'fused' or 'collective'")
        self.reduce = reduce
        self.overlap = overlap

    def make_optimizer(self, model: torch.nn.Module, cfg):
        if self.reduce == "fused" and next(model.parameters()).dtype != torch.bfloat16:
            self.reduce = "collective"  # the peer-memory path exchanges bf16 weights and gradients
        if self.reduce == "fused" and self.overlap:
            from .fsdp import FSDPAdamW

            return FSDPAdamW(model, cfg, self.group, fused=True, reshard=False, replicate_units=True,
                             overlap=True)
        if self.reduce == "fused":
            return FusedDPAdamW(model, cfg, self.group)
        opt = DPFusedAdamW(model.parameters(), lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                           weight_decay=cfg.weight_decay, max_grad_norm=cfg.grad_clip,
                           world_size=self.world,
                           use_kernels=getattr(getattr(model, "config", None), "use_kernels", None))
        src = dist.get_global_rank(self.group, 0) if self.group else 0
        dist.broadcast(opt.space.flat, src=src, group=self.group)
        if opt.master is not opt.space.flat:
            opt.master.copy_(opt.space.flat)
        for b in model.buffers():
            dist.broadcast(b, src=src, group=self.group)
        return opt

    def reduce_gradients(self, optimizer) -> None:
        """Agree on the set of parameters that received gradients; sum the gradients
        (collective path) -- the fused path reduces inside its optimizer step."""
        # The set is a property of the model structure, so it is agreed once (a small
        # all-reduce + host read) and reused while the local set is unchanged.
        local = tuple(optimizer.space.got)
        if local != getattr(self, "_last_local", None):
            got = torch.tensor(local, dtype=torch.uint8, device=optimizer.space.device)
            dist.all_reduce(got, op=dist.ReduceOp.MAX, group=self.group)
            self._last_local = local
            self._agreed = [bool(x) for x in got.tolist()]
        optimizer.space.got = list(self._agreed)
        if self.reduce == "collective":
            dist.all_reduce(optimizer.space.grad, group=self.group)
