"""Fully sharded data parallelism: parameters sharded per block, all-gathered in
the forward (fused into a tensor-core GEMM), gradients reduce-scattered.

The reference shards with PyTorch FSDP through Accelerate
(`scripts/pretrain_distributed.py:24`, `configs/fsdp_config.yaml`): every
wrapped unit all-gathers its parameters before use and reduce-scatters its
gradients.  Here one process drives one GPU and the exchange runs in kernels
over NVLink peer memory (``csrc/gemm_tc.cu``, ``csrc/comm.cu``):

* Layout.  The flat parameter buffer (bf16, same layout on every rank) holds
  the replicated group first (embedding, norms, persistent tokens, gate and
  conv parameters: everything that is not an ``nn.Linear`` weight of a block),
  then one unit per block with that block's ``nn.Linear`` weights.  Each group
  is split evenly over the ranks (8-element aligned); rank r keeps the fp32
  master copy and AdamW moments of its part of every group.
* Step.  One bounded barrier (all backwards done), a reduce-scatter in which
  each rank sums its parts of the gradient from every rank's buffer (peer
  loads) and publishes its squared norm, a second barrier, then AdamW on the
  shard with the global clip.  New replicated values are stored into every
  rank's buffer; new unit values only into this rank's (the unit is sharded
  until its next use).  A third barrier closes the step.
* Forward.  A block's forward pre-hook gathers its unit if that has not
  happened since the last step.  The block's first ``ops.linear`` call runs
  the fused kernel: the GEMM on the block's weights (tcgen05, this GPU's
  memory) while a gather warp per CTA streams the NEXT block's unit from the
  owners into this rank's buffer, so the all-gather is hidden under the
  tensor-core tiles and the next block finds its parameters in place.  The
  first block's unit is gathered by the standalone gather kernel.
* The gathered parameters stay in place through the backward (the gradient
  GEMMs read local memory), as in FSDP's SHARD_GRAD_OP mode; on a 180 GB GPU the
  bf16 parameters are 1/8 of the per-parameter bytes (fp32 master and two
  moments are the sharded bulk).

``reduce="collective"`` (CPU / gloo, and the baseline) runs the same layout
with ``torch.distributed`` collectives: all-reduce of the gradient, the shard
update in PyTorch, and ``all_gather`` for the gathers.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops import linear as linear_ops
from ..ops._ext import ext
from ..train.optim import ALIGN, FlatParamSpace, FusedAdamW, segment_table, unique_trainable
from .ddp import _PeerBuffer


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


def shard_units(model: nn.Module):
    """Parameter order and units: ``(params, unit_modules, unit_param_lists)``.

    The replicated parameters come first; each block of ``model.blocks``
    contributes one unit holding its ``nn.Linear`` weights."""
    all_params = unique_trainable(model.parameters())
    taken: set[int] = set()
    units, unit_params = [], []
    for block in getattr(model, "blocks", []):
        ps = []
        for m in block.modules():
            if isinstance(m, nn.Linear) and m.weight.requires_grad and id(m.weight) not in taken:
                ps.append(m.weight)
                taken.add(id(m.weight))
        if ps:
            units.append(block)
            unit_params.append(ps)
    replicated = [p for p in all_params if id(p) not in taken]
    ordered = replicated + [p for ps in unit_params for p in ps]
    return ordered, units, unit_params


class ShardLayout:
    """Groups of the flat buffer and each rank's part of them.

    ``groups``: list of ``(flat_offset, length, shard, replicated, shard_offset)``;
    rank r owns group-relative ``[r * shard, min((r + 1) * shard, length))``
    stored at ``shard_offset`` of its optimizer shard."""

    def __init__(self, ranges: list[tuple[int, int, bool]], world: int) -> None:
        self.world = world
        self.groups = []
        off = 0
        for a, n, repl in ranges:
            s = max(8, _round8(-(-n // world)))
            self.groups.append((a, n, s, repl, off))
            off += s
        self.n_shard = off

    def owned(self, rank: int):
        """(flat_offset, shard_offset, length, replicated) of rank's valid parts."""
        out = []
        for a, n, s, repl, so in self.groups:
            lo = rank * s
            ln = min(s, n - lo)
            if ln > 0:
                out.append((a + lo, so, ln, repl))
        return out

    def update_segments(self, active: list[tuple[int, int]], rank: int):
        """Active flat ranges clipped to the rank's parts: (shard_offset, length, flat - shard, replicated)."""
        out = []
        for fo, so, ln, repl in self.owned(rank):
            for o, n in active:
                lo, hi = max(o, fo), min(o + n, fo + ln)
                if lo < hi:
                    out.append((so + lo - fo, hi - lo, fo - so, repl))
        out.sort()
        return out


class FSDPAdamW(FusedAdamW):
    """AdamW over per-block parameter shards; see the module docstring."""

    # each rank holds only its shard of the optimizer state: checkpoints keep one file per rank
    shard_state = True

    def __init__(self, model: nn.Module, cfg, group=None, fused: bool = True):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.fused = fused
        params, units, unit_params = shard_units(model)
        device = params[0].device
        if fused and params[0].dtype != torch.bfloat16:
            raise ValueError("the fused sharded path runs bf16 parameters")
        self._bufs = []

        def peer_buffers(total, dtype):
            fb = _PeerBuffer(total * 2, device, group, self.world, self.rank)
            gb = _PeerBuffer(total * 2, device, group, self.world, self.rank)
            self._bufs += [fb, gb]
            self._param_buf, self._grad_buf = fb, gb
            return fb.local.view(torch.bfloat16), gb.local.view(torch.bfloat16)

        space = FlatParamSpace(params, pad_to=ALIGN, buffers=peer_buffers if fused else None)
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast(space.flat, src=src, group=group)
        for b in model.buffers():
            dist.broadcast(b, src=src, group=group)
        torch.optim.Optimizer.__init__(self, space.params, dict(lr=cfg.lr, betas=tuple(cfg.betas), eps=cfg.eps,
                                                                 weight_decay=cfg.weight_decay))
        self.space = space
        self.max_grad_norm = float(cfg.grad_clip)
        self.kernels = fused
        self.step_count = 0
        # groups: replicated [0, first unit offset), then one per unit
        pos = {id(p): i for i, p in enumerate(space.params)}
        ends = [o + (p.numel() + ALIGN - 1) // ALIGN * ALIGN for p, o in zip(space.params, space.offsets)]
        ranges, self.unit_ranges = [], []
        first = space.offsets[pos[id(unit_params[0][0])]] if unit_params else space.total
        if first > 0:
            ranges.append((0, first, True))
        for ps in unit_params:
            idx = [pos[id(p)] for p in ps]
            a, b = space.offsets[min(idx)], ends[max(idx)]
            ranges.append((a, b - a, False))
        self.layout = ShardLayout(ranges, self.world)
        self.unit_groups = [g for g in self.layout.groups if not g[3]]
        self.units = units
        n = self.layout.n_shard
        self.master = torch.zeros(n, dtype=torch.float32, device=device)
        for fo, so, ln, _ in self.layout.owned(self.rank):
            self.master[so:so + ln].copy_(space.flat[fo:fo + ln])
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=device)
        self.gsum = torch.zeros(n, dtype=torch.float32, device=device)
        self.norm_out = torch.zeros(1, dtype=torch.float32, device=device)
        self.last_grad_norm = self.norm_out
        self.stale = [False] * len(units)  # every rank holds the full parameters after the broadcast
        self._tab_key = None
        self.graph_safe = fused
        if fused:
            self.sig = _PeerBuffer(4 * 4 * self.world, device, group, self.world, self.rank)
            self.slots = _PeerBuffer(4 * self.world, device, group, self.world, self.rank)
            self._bufs += [self.sig, self.slots]
            self.err = torch.zeros(1, dtype=torch.int32, device=device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
            owned = self.layout.owned(self.rank)
            rt = torch.empty(4 * len(owned), dtype=torch.long)
            items = 0
            for i, (fo, so, ln, _) in enumerate(owned):
                rt[3 * i], rt[3 * i + 1], rt[3 * i + 2], rt[3 * len(owned) + i] = fo, so, ln, items
                items += (ln + (1 << 14) - 1) // (1 << 14)
            self._rtab = (rt.to(device), len(owned), items)
        self._hooks = [m.register_forward_pre_hook(self._make_pre_hook(u)) for u, m in enumerate(units)]

    # ------------------------------------------------------------ gathers
    def grad_scale(self) -> float:
        return 1.0 / self.world

    def _gather(self, u: int) -> None:
        a, n, s, _, _ = self.unit_groups[u]
        if self.fused:
            ext().fsdp_gather(self.space.flat, self._param_buf.ptrs, a, n, s, self.rank)
        else:
            self._gather_collective(a, n, s)
        self.stale[u] = False

    def _gather_collective(self, a: int, n: int, s: int) -> None:
        flat = self.space.flat
        lo = self.rank * s
        mine = torch.zeros(s, dtype=flat.dtype, device=flat.device)
        ln = max(0, min(s, n - lo))
        if ln:
            mine[:ln].copy_(flat[a + lo:a + lo + ln])
        parts = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(parts, mine, group=self.group)
        flat[a:a + n].copy_(torch.cat(parts)[:n])

    def _make_pre_hook(self, u: int):
        def hook(_module, _args):
            if self.world == 1:
                return None
            if self.stale[u]:
                self._gather(u)
            nxt = u + 1
            if self.fused and nxt < len(self.units) and self.stale[nxt]:
                linear_ops.set_prefetch(self._prefetcher(nxt))
            else:
                linear_ops.set_prefetch(None)
            return None
        return hook

    def _prefetcher(self, u: int):
        a, n, s, _, _ = self.unit_groups[u]

        def run(x: torch.Tensor, w: torch.Tensor):
            K = x.shape[-1]
            N = w.shape[0]
            if (not x.is_cuda or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.numel() == 0
                    or K % 8 or N % 8 or not self.stale[u]):
                return None
            x2 = x.reshape(-1, K)
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            y = ext().gemm_gather_tc(x2, w.contiguous(), self.space.flat, self._param_buf.ptrs, a, n, s,
                                     self.rank, False)
            self.stale[u] = False
            return y.view(*x.shape[:-1], N)
        return run

    def materialize(self) -> None:
        """Gather every unit that is still sharded (before saving or reading parameters directly)."""
        linear_ops.set_prefetch(None)
        for u in range(len(self.units)):
            if self.stale[u]:
                self._gather(u)

    # ------------------------------------------------------------ step
    def _update_table(self):
        segs = self.space.active_segments()
        key = tuple(segs)
        if key != self._tab_key:
            upd = self.layout.update_segments(segs, self.rank)
            self._upd = upd
            tab, nseg, items = segment_table([(o, ln) for o, ln, _, _ in upd], self.space.device)
            aux = torch.tensor([v for _, _, d, r in upd for v in (d, int(r))] or [0], dtype=torch.long)
            self._tab = (tab, nseg, items, aux.to(self.space.device))
            self._tab_key = key
        return self._tab

    @torch.no_grad()
    def step(self, closure=None, hyper: torch.Tensor | None = None, schedule: tuple | None = None):
        loss = closure() if closure is not None else None
        linear_ops.set_prefetch(None)
        self.step_count += 1
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        tab, nseg, items, aux = self._update_table()
        if self.fused:
            E = ext()
            w, me = self.world, self.rank
            if hyper is not None:
                warm, total, mr = schedule if schedule is not None else (0, 1, 1.0)
                E.adamw_hyper_step(hyper, g.get("initial_lr", lr), b1, b2, warm, total, mr, schedule is not None)
            E.comm_barrier(self.sig.ptrs, 0, self.epoch, True, w, me, self.err)   # all gradients complete
            rt, rn, ri = self._rtab
            E.comm_reduce_segments(self._grad_buf.ptrs, rt, rn, ri, self.gsum, self.grad_scale(),
                                   self.slots.ptrs, w, me)
            E.comm_barrier(self.sig.ptrs, 1, self.epoch, False, w, me, self.err)  # all shard norms published
            E.comm_adamw_shard(self.gsum, self.master, self.exp_avg, self.exp_avg_sq, self._param_buf.ptrs, 0, w,
                               tab, nseg, items, self.slots.local.view(torch.float32), self.grad_scale(),
                               self.max_grad_norm, lr, b1, b2, eps, wd, self.step_count, self.norm_out, hyper,
                               aux, me)
            E.comm_barrier(self.sig.ptrs, 2, self.epoch, False, w, me, self.err)  # every rank's shard written
        else:
            self._step_collective(lr, b1, b2, eps, wd)
        if self.world > 1:
            self.stale = [True] * len(self.units)
        return loss

    def _step_collective(self, lr, b1, b2, eps, wd):
        s = self.space
        dist.all_reduce(s.grad, group=self.group)
        gs = self.grad_scale()
        owned = self.layout.owned(self.rank)
        if s.dtype == torch.float32:
            # fp32 parameters are their own master copy (as in the one-process optimizer), so
            # values a forward wrote into parameter storage (MAC's memory state) are kept
            for fo, so, ln, _ in owned:
                self.master[so:so + ln].copy_(s.flat[fo:fo + ln])
        for fo, so, ln, _ in owned:
            self.gsum[so:so + ln].copy_(s.grad[fo:fo + ln].float())
        coef = 1.0
        if self.max_grad_norm > 0:
            sq = torch.zeros(1, dtype=torch.float64, device=s.device)
            for _, so, ln, _ in owned:
                sq += (self.gsum[so:so + ln].double() * gs).pow(2).sum()
            dist.all_reduce(sq, group=self.group)
            nrm = math.sqrt(float(sq))
            self.norm_out.fill_(nrm)
            coef = min(1.0, self.max_grad_norm / (nrm + 1e-6))
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        for so, ln, delta, _ in self._upd:
            gr = self.gsum[so:so + ln] * (gs * coef)
            p, m, v = self.master[so:so + ln], self.exp_avg[so:so + ln], self.exp_avg_sq[so:so + ln]
            p.mul_(1 - lr * wd)
            m.mul_(b1).add_(gr, alpha=1 - b1)
            v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            p.addcdiv_(m, v.sqrt().div_(math.sqrt(bc2)).add_(eps), value=-lr / bc1)
            s.flat[so + delta:so + delta + ln].copy_(p)
        # the replicated group is all-gathered now; units when next used
        for a, n, sh, repl, _ in self.layout.groups:
            if repl:
                self._gather_collective(a, n, sh)

    def check_errors(self) -> None:
        if self.fused:
            v = int(self.err.item())
            if v:
                raise RuntimeError(f"sharded data-parallel step: cross-GPU wait timed out (code {v})")

    def state_dict(self):
        return {"step": self.step_count, "rank": self.rank, "world": self.world, "n_shard": self.layout.n_shard,
                "master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq,
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, sd):
        if (int(sd["world"]), int(sd["rank"]), int(sd["n_shard"])) != (self.world, self.rank, self.layout.n_shard):
            raise ValueError("optimizer shard layout differs (world size or model changed?)")
        self.step_count = int(sd["step"])
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for pg, sg in zip(self.param_groups, sd["param_groups"]):
            pg.update(sg)

    def close(self):
        linear_ops.set_prefetch(None)
        for h in self._hooks:
            h.remove()
        self._hooks = []
        for b in self._bufs:
            b.close()


class FullyShardedEngine:
    """Engine for :class:`~titans_pytorch_b200.train.trainer.Trainer` (``engine=``)."""

    def __init__(self, group=None, reduce: str | None = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("FullyShardedEngine needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if reduce is None:
            reduce = "fused" if (torch.cuda.is_available() and dist.get_backend(group) == "nccl") else "collective"
        if reduce not in ("fused", "collective"):
            raise ValueError("reduce must be 'fused' or 'collective'")
        self.reduce = reduce

    def make_optimizer(self, model: nn.Module, cfg):
        fused = self.reduce == "fused" and next(model.parameters()).dtype == torch.bfloat16
        self.reduce = "fused" if fused else "collective"
        return FSDPAdamW(model, cfg, self.group, fused=fused)

    def reduce_gradients(self, optimizer) -> None:
        """Agree on the set of parameters that received gradients (the reduction
        itself runs inside the optimizer step)."""
        local = tuple(optimizer.space.got)
        if local != getattr(self, "_last_local", None):
            got = torch.tensor(local, dtype=torch.uint8, device=optimizer.space.device)
            dist.all_reduce(got, op=dist.ReduceOp.MAX, group=self.group)
            self._last_local = local
            self._agreed = [bool(x) for x in got.tolist()]
        optimizer.space.got = list(self._agreed)


__all__ = ["FullyShardedEngine", "FSDPAdamW", "ShardLayout", "shard_units"]
