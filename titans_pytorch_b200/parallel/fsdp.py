"""Sharded data parallelism over NVLink peer memory: per-block parameter
shards, gradients reduce-scattered during the backward, and (FSDP) parameters
gathered for each use and dropped afterwards.

The reference shards with PyTorch FSDP through Accelerate
(`scripts/pretrain_distributed.py:24`, `configs/fsdp_config.yaml`; DDP at
`:350-413`): every wrapped unit all-gathers its parameters before use and
reduce-scatters its gradients, and DDP all-reduces gradient buckets from
autograd hooks while the backward runs.  Here one process drives one GPU and
the exchange runs in kernels over peer memory (``csrc/comm.cu``,
``csrc/gemm_tc.cu``):

* Units and shards.  The replicated group holds everything that is not an
  ``nn.Linear`` weight of a block (embedding, norms, persistent tokens, gate
  and conv parameters, and MAC's memory-MLP weights, which its forward
  overwrites with the memory state); each block's ``nn.Linear`` weights form
  one unit.  Every group is split evenly over the ranks (8-element aligned);
  rank r keeps the fp32 master copy and AdamW moments of its part of every
  group.
* Calls.  A forward runs the blocks in some order (MAC runs every block once
  per segment); call c is the c-th block forward of a forward pass.  Its
  output tensor gets a hook that fires in the backward just before the
  call's own backward, so when it fires every later call's backward is
  complete.
* Reduction during the backward.  When a call's (or, without resharding, a
  unit's last call's) backward is complete, a communication stream waits for
  it, passes a bounded cross-GPU barrier (every rank done with it), and runs
  the peer-load reduce of this rank's part of the unit into the fp32 shard
  gradient, with the block partials of the squared norm.  The tensor cores
  meanwhile run the backward of the earlier calls.  The replicated group is
  reduced at the step; then the norm is published, and AdamW stores the new
  bf16 values: replicated parameters into every rank's buffer, units into
  every rank's buffer (``replicate_units``: data parallelism), into this
  rank's flat buffer (sharded, gathered at the next forward), or into this
  rank's shard store (``reshard``).
* ``reshard`` (FULL_SHARD).  A unit's parameters and gradients live in a ring
  of R working slots: call c binds its unit's parameters and gradients to
  slot c mod R (so R units are resident at a time, not all of them).  The
  unit is gathered from the owners' shard stores into the slot before the
  call (the previous call's first GEMM streams it in: ``gemm_gather_tc``, the
  all-gather fused into the tensor-core GEMM), gathered again before the
  call's backward (on a second stream while the later call's backward runs),
  and its gradient is reduce-scattered right after the call's backward, with
  a second barrier before the slot is reused.  Over several calls or
  micro-batches a unit's reductions accumulate in the fp32 shard gradient.
* Without ``reshard`` (SHARD_GRAD_OP; and data parallelism) the flat buffers
  are full size and a unit is reduced once its last call is done.

``reduce="collective"`` (CPU / gloo) runs the same layout and hooks with
``torch.distributed`` collectives (all-gather of units, all-reduce of each
reduced range); it is the path the CPU tests compare with one process.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops import linear as linear_ops
from ..ops._ext import ext
from ..train.optim import ALIGN, FlatParamSpace, FusedAdamW, segment_table, unique_trainable
from .peer import PeerBuffer

CHUNK = 1 << 14  # elements per work item of the reduce / update kernels
OVERLAP_CTAS = 16  # CTAs of a reduce that runs during the backward


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


def _in_backward() -> bool:
    """True inside an autograd backward (e.g. a checkpointed block's recompute)."""
    f = getattr(torch._C, "_current_autograd_node", None)
    return f is not None and f() is not None


def _memory_state_weights(model: nn.Module) -> set[int]:
    """Weights a forward overwrites (MAC writes the memory state into its memory MLP)."""
    if getattr(model, "model_type", "") != "mac":
        return set()
    from ..models.memory import MemoryMLP

    return {id(p) for m in model.modules() if isinstance(m, MemoryMLP) for p in m.parameters()}


def shard_units(model: nn.Module):
    """Parameter order and units: ``(params, unit_modules, unit_param_lists)``.

    The replicated parameters come first; each block of ``model.blocks``
    contributes one unit holding its ``nn.Linear`` weights (minus weights the
    forward writes into)."""
    all_params = unique_trainable(model.parameters())
    keep_replicated = _memory_state_weights(model)
    taken: set[int] = set()
    units, unit_params = [], []
    for block in getattr(model, "blocks", []):
        ps = []
        for m in block.modules():
            w = getattr(m, "weight", None)
            if (isinstance(m, nn.Linear) and w.requires_grad and id(w) not in taken
                    and id(w) not in keep_replicated):
                ps.append(w)
                taken.add(id(w))
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
    """AdamW over per-block parameter shards; see the module docstring.

    ``reshard``: FULL_SHARD (working slots, per-call gathers and reductions);
    ``replicate_units``: data parallelism (new unit values stored on every
    rank, nothing gathered); ``overlap``: reductions on a communication stream
    during the backward (fused path); ``slots``: working slots with ``reshard``."""

    # each rank holds only its shard of the optimizer state: checkpoints keep one file per rank
    shard_state = True

    def __init__(self, model: nn.Module, cfg, group=None, fused: bool = True, reshard: bool = False,
                 replicate_units: bool = False, overlap: bool = True, slots: int = 3):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.fused = fused
        params, units, unit_params = shard_units(model)
        device = params[0].device
        dtype = params[0].dtype
        if fused and dtype != torch.bfloat16:
            raise ValueError("the fused sharded path runs bf16 parameters")
        self.reshard = bool(reshard) and bool(units) and not replicate_units
        self.replicate_units = bool(replicate_units)
        self.overlap = bool(overlap)
        self.units = units
        self.unit_params = unit_params

        # ---------------------------------------------------------- logical layout
        sizes = [(p.numel() + ALIGN - 1) // ALIGN * ALIGN for p in params]
        offsets, off = [], 0
        for n in sizes:
            offsets.append(off)
            off += n
        total_logical = off
        pos = {id(p): i for i, p in enumerate(params)}
        self.unit_range = []  # (logical start, length)
        for ps in unit_params:
            idx = [pos[id(p)] for p in ps]
            a, b = offsets[min(idx)], offsets[max(idx)] + sizes[max(idx)]
            self.unit_range.append((a, b - a))
        first = self.unit_range[0][0] if units else total_logical
        ranges = [(0, first, True)] if first > 0 else []
        ranges += [(a, n, False) for a, n in self.unit_range]
        self.layout = ShardLayout(ranges, self.world)
        self.n_rep = first
        self.rep_group = self.layout.groups[0] if first > 0 else None
        self.unit_groups = [g for g in self.layout.groups if not g[3]]
        n_shard = self.layout.n_shard

        # ---------------------------------------------------------- physical layout
        if self.reshard:
            self.R = max(2, min(int(slots), len(units)))
            self.max_n = max(n for _, n in self.unit_range)
            self.slot_base = [first + k * self.max_n for k in range(self.R)]
            phys_total = first + self.R * self.max_n
            unit_of = {}
            for u, ps in enumerate(unit_params):
                for p in ps:
                    unit_of[id(p)] = u
            phys = []
            for p, o in zip(params, offsets):
                u = unit_of.get(id(p))
                phys.append(o if u is None else self.slot_base[0] + o - self.unit_range[u][0])
            placement = (phys, phys_total)
            self.S_base = phys_total  # shard store follows the flat part of the parameter buffer
            p_total = phys_total + n_shard
        else:
            self.R = len(units)
            phys_total = total_logical
            placement = None
            self.S_base = 0
            p_total = phys_total

        # ---------------------------------------------------------- initial values (same on every rank)
        src = dist.get_global_rank(group, 0) if group is not None else 0
        logical = torch.empty(total_logical, dtype=dtype, device=device)
        with torch.no_grad():
            for p, o in zip(params, offsets):
                logical[o:o + p.numel()].copy_(p.detach().reshape(-1))
        dist.broadcast(logical, src=src, group=group)
        for b in model.buffers():
            dist.broadcast(b, src=src, group=group)

        self._bufs = []
        if fused:
            def peer_buffers(total, dt):
                pb = PeerBuffer(p_total * 2, device, group, self.world, self.rank)
                gb = PeerBuffer(total * 2, device, group, self.world, self.rank)
                self._bufs += [pb, gb]
                self._param_buf, self._grad_buf = pb, gb
                self._P = pb.local.view(torch.bfloat16)
                return self._P[:total], gb.local.view(torch.bfloat16)

            space = FlatParamSpace(params, buffers=peer_buffers, placement=placement)
        else:
            space = FlatParamSpace(params, placement=placement)
            self._P = None
        with torch.no_grad():
            if self.reshard:
                space.flat[:first].copy_(logical[:first])
            else:
                space.flat[:total_logical].copy_(logical)
        torch.optim.Optimizer.__init__(self, space.params, dict(lr=cfg.lr, betas=tuple(cfg.betas), eps=cfg.eps,
                                                                 weight_decay=cfg.weight_decay))
        self.space = space
        self.max_grad_norm = float(cfg.grad_clip)
        self.kernels = fused
        self.step_count = 0
        self.master = torch.zeros(n_shard, dtype=torch.float32, device=device)
        for fo, so, ln, _ in self.layout.owned(self.rank):
            self.master[so:so + ln].copy_(logical[fo:fo + ln])
        if self.reshard:  # this rank's part of every unit, in bf16 (the gathers' source)
            self.store = self._P[self.S_base:self.S_base + n_shard] if fused else \
                torch.zeros(n_shard, dtype=dtype, device=device)
            for fo, so, ln, repl in self.layout.owned(self.rank):
                if not repl:
                    self.store[so:so + ln].copy_(logical[fo:fo + ln])
        del logical
        self.exp_avg = torch.zeros(n_shard, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(n_shard, dtype=torch.float32, device=device)
        self.gsum = torch.zeros(n_shard, dtype=torch.float32, device=device)
        self.norm_out = torch.zeros(1, dtype=torch.float32, device=device)
        self.last_grad_norm = self.norm_out
        self._tab_key = None
        self.graph_safe = fused
        # per-call / per-block reductions read the gradients inside the backward
        self.reduces_during_backward = self.reshard or (self.overlap and fused) or not self.replicate_units

        # ---------------------------------------------------------- reduction tables
        w, me = self.world, self.rank
        self._nsm = torch.cuda.get_device_properties(device).multi_processor_count if device.type == "cuda" else 1
        self._part_off, nparts = [], 0
        self._blocks = []
        for a, n, s, repl, so in self.layout.groups:
            ln = max(0, min(s, n - me * s))
            items = (ln + CHUNK - 1) // CHUNK
            # a unit's reduce runs beside the backward's persistent GEMMs: a few CTAs
            # stream it in the background instead of taking SMs from the tensor cores
            cap = OVERLAP_CTAS if (self.overlap and fused and not repl) else 2 * self._nsm
            blocks = max(1, min(items, cap))
            self._part_off.append(nparts)
            self._blocks.append((ln, items, blocks))
            nparts += blocks
        self._nparts = nparts
        self.part = torch.zeros(max(1, nparts), dtype=torch.float32, device=device)
        gi0 = 1 if self.rep_group is not None else 0  # layout group index of unit 0

        def table(base, gi):
            a, n, s, repl, so = self.layout.groups[gi]
            ln = self._blocks[gi][0]
            segs = [(base + me * s, so, ln)] if ln > 0 else []
            t = torch.empty(max(1, 4 * len(segs)), dtype=torch.long)
            for j, (fo, soff, lnn) in enumerate(segs):
                t[3 * j], t[3 * j + 1], t[3 * j + 2], t[3 * len(segs) + j] = fo, soff, lnn, 0
            return t.to(device), len(segs)

        self._gi = [gi0 + u for u in range(len(units))]
        self._rep_tab = table(0, 0) if self.rep_group is not None else None
        if self.reshard:
            self._unit_tab = [[table(self.slot_base[k], self._gi[u]) for k in range(self.R)]
                              for u in range(len(units))]
        else:
            self._unit_tab = [[table(self.unit_range[u][0], self._gi[u])] for u in range(len(units))]

        # ---------------------------------------------------------- peer signalling, streams, gathers
        if fused:
            self.sig = PeerBuffer(4 * 4 * w, device, group, w, me)
            self.slots_buf = PeerBuffer(4 * w, device, group, w, me)
            self._bufs += [self.sig, self.slots_buf]
            self.err = torch.zeros(1, dtype=torch.int32, device=device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=device)    # step barriers 0-2
            self.epoch_u = torch.zeros(1, dtype=torch.int32, device=device)  # per-call barriers (slot 3)
            self._rs = torch.cuda.Stream(device) if self.overlap else None   # reductions
            self._gs = torch.cuda.Stream(device)                             # backward re-gathers
            if self.reshard:
                # owner r keeps unit element e (r*s <= e < (r+1)*s) at store_r[so + e - r*s]; the
                # gather kernels read src[r] + u0 + e, so src[r] = P_r + S_base + so - r*s - u0
                self._src = []
                for u in range(len(units)):
                    _, n, s, _, so = self.layout.groups[self._gi[u]]
                    per = []
                    for k in range(self.R):
                        ptrs = [pr + 2 * (self.S_base + so - r * s - self.slot_base[k])
                                for r, pr in enumerate(self._param_buf.host_ptrs)]
                        per.append(torch.tensor(ptrs, dtype=torch.int64, device=device))
                    self._src.append(per)
        # ---------------------------------------------------------- host state machine
        self.stale = [False] * len(units)  # (no reshard) every rank holds the full parameters now
        self._calls: list[int] = []      # unit of each call of the current forward
        self._seq: list[int] = []        # the previous forward's calls (prefetch prediction)
        self._phase = "idle"
        self._done_above = 0             # calls >= this have finished their backward
        self._reduced: set[int] = set()  # units reduced at least once this step
        self._unit_reduced = [False] * len(units)
        self._armed = True
        self._rs_used = self._gs_used = False
        self._main = torch.cuda.current_stream(device) if fused else None
        self._slot_unit = [-1] * self.R if self.reshard else []
        self._bound = [-1] * len(units)
        self._gather_evt = [None] * self.R if self.reshard else []
        self._gslot_evt = [None] * self.R if self.reshard else []
        self._gslot_dirty = [False] * self.R if self.reshard else []
        self._hooks = [model.register_forward_pre_hook(lambda m, a: self._begin_forward())]
        for u, m in enumerate(units):
            self._hooks.append(m.register_forward_pre_hook(self._make_pre_hook(u)))
            self._hooks.append(m.register_forward_hook(self._make_post_hook(u)))

    # ------------------------------------------------------------ sizes
    def comm_bytes(self) -> int:
        """Device bytes held outside PyTorch's allocator (the peer-visible buffers)."""
        return sum(b.nbytes for b in self._bufs)

    def grad_scale(self) -> float:
        return 1.0 / self.world

    # ------------------------------------------------------------ binding (reshard)
    def _bind(self, u: int, k: int) -> None:
        """Point unit u's parameters and gradients at working slot k."""
        if self._bound[u] == k:
            return
        s = self.space
        a = self.unit_range[u][0]
        base = self.slot_base[k]
        idx = self._param_index()
        for p in self.unit_params[u]:
            o = base + s.offsets[idx[id(p)]] - a
            n = p.numel()
            p.data = s.flat[o:o + n].view_as(p)
            p.grad = s.grad[o:o + n].view_as(p)
        self._bound[u] = k

    def _param_index(self):
        if not hasattr(self, "_pidx"):
            self._pidx = {id(p): i for i, p in enumerate(self.space.params)}
        return self._pidx

    # ------------------------------------------------------------ gathers
    def _gather(self, u: int, k: int | None = None) -> None:
        """Unit u into working slot k (reshard) or into its flat range (sharded in place)."""
        gi = self._gi[u]
        a, n, s, _, so = self.layout.groups[gi]
        if self.reshard:
            if self.fused:
                ext().fsdp_gather(self._P, self._src[u][k], self.slot_base[k], n, s, self.rank, True)
            else:
                self._gather_collective(self.store[so:so + s], self.space.flat, self.slot_base[k], n, s)
            return
        if self.fused:
            ext().fsdp_gather(self.space.flat, self._param_buf.ptrs, a, n, s, self.rank)
        else:
            lo = self.rank * s
            ln = max(0, min(s, n - lo))
            mine = torch.zeros(s, dtype=self.space.flat.dtype, device=self.space.flat.device)
            if ln:
                mine[:ln].copy_(self.space.flat[a + lo:a + lo + ln])
            self._gather_collective(mine, self.space.flat, a, n, s)
        self.stale[u] = False

    def _gather_collective(self, mine: torch.Tensor, dst: torch.Tensor, at: int, n: int, s: int) -> None:
        part = torch.zeros(s, dtype=dst.dtype, device=dst.device)
        part[:mine.numel()].copy_(mine[:s])
        parts = [torch.empty_like(part) for _ in range(self.world)]
        dist.all_gather(parts, part, group=self.group)
        dst[at:at + n].copy_(torch.cat(parts)[:n])

    def _prefetcher(self, u: int, k: int | None):
        """One-shot GEMM hook: the next ``linear`` call also gathers unit u (into slot k)."""
        a, n, s, _, _ = self.layout.groups[self._gi[u]]

        def run(x: torch.Tensor, w: torch.Tensor):
            K, N = x.shape[-1], w.shape[0]
            if (not x.is_cuda or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or x.numel() == 0
                    or K % 8 or N % 8):
                return None
            if self.reshard:
                if self._slot_unit[k] == u:
                    return None
            elif not self.stale[u]:
                return None
            x2 = x.reshape(-1, K)
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            if self.reshard:
                y = ext().gemm_gather_tc(x2, w.contiguous(), self._P, self._src[u][k], self.slot_base[k], n, s,
                                         self.rank, False, True)
                self._slot_unit[k] = u
            else:
                y = ext().gemm_gather_tc(x2, w.contiguous(), self.space.flat, self._param_buf.ptrs, a, n, s,
                                         self.rank, False)
                self.stale[u] = False
            return y.view(*x.shape[:-1], N)
        return run

    def materialize(self) -> None:
        """Gather every unit that is still sharded (not available with ``reshard``:
        use :meth:`full_model_state_dict`)."""
        linear_ops.set_prefetch(None)
        if self.reshard:
            return
        for u in range(len(self.units)):
            if self.stale[u]:
                self._gather(u)

    @torch.no_grad()
    def full_model_state_dict(self, model: nn.Module) -> dict[str, torch.Tensor]:
        """``model.state_dict()`` with every unit's current values (gathered one at a
        time into a working slot), on the host."""
        linear_ops.set_prefetch(None)
        self._join()
        sd = {k: v.detach().cpu() for k, v in model.state_dict().items()}
        if not self.reshard:
            self.materialize()
            return {k: v.detach().cpu() for k, v in model.state_dict().items()}
        names: dict[int, list[str]] = {}
        for name, p in model.named_parameters(remove_duplicate=False):
            names.setdefault(id(p), []).append(name)
        for u in range(len(self.units)):
            self._bind(u, 0)
            self._gather(u, 0)
            self._slot_unit[0] = u
            for p in self.unit_params[u]:
                v = p.detach().cpu().clone()
                for name in names.get(id(p), []):
                    sd[name] = v
        return sd

    # ------------------------------------------------------------ hooks
    def prepare_backward(self, last_micro: bool) -> None:
        """Called by the trainer before each backward: without resharding the
        reductions run only for the last micro-batch of a step (the gradients
        accumulate in place until then)."""
        self._armed = self.reshard or bool(last_micro)

    def _begin_forward(self) -> None:
        if _in_backward():
            return
        if self._phase in ("backward", "flushed"):
            # another micro-batch: its backward accumulates into the same flat gradients, so
            # (without resharding) the reductions of this one are redone over the sum
            self._flush()
            if not self.reshard:
                self._unit_reduced = [False] * len(self.units)
        if self._calls:
            self._seq = self._calls
        self._calls = []
        self._phase = "forward"
        if self.fused:
            self._main = torch.cuda.current_stream(self.space.device)  # the stream the backward follows
            if self._gs_used:
                self._main.wait_stream(self._gs)
                self._gs_used = False

    def _make_pre_hook(self, u: int):
        def hook(_module, _args):
            if _in_backward():  # recompute of a checkpointed block: its backward hook prepared the call
                return None
            c = len(self._calls)
            self._calls.append(u)
            if self.reshard:
                k = c % self.R
                self._bind(u, k)
                if self._slot_unit[k] != u:
                    self._gather(u, k)
                    self._slot_unit[k] = u
                nxt = self._seq[c + 1] if c + 1 < len(self._seq) else None
                k2 = (c + 1) % self.R
                if self.fused and nxt is not None and nxt != u and k2 != k and self._slot_unit[k2] != nxt:
                    linear_ops.set_prefetch(self._prefetcher(nxt, k2))
                else:
                    linear_ops.set_prefetch(None)
                return None
            if self.world == 1 or self.replicate_units:
                return None
            if self.stale[u]:
                self._gather(u)
            nxt = u + 1
            if self.fused and nxt < len(self.units) and self.stale[nxt]:
                linear_ops.set_prefetch(self._prefetcher(nxt, None))
            else:
                linear_ops.set_prefetch(None)
            return None
        return hook

    def _make_post_hook(self, u: int):
        def hook(_module, _args, out):
            if _in_backward() or not torch.is_grad_enabled():
                return None
            c = len(self._calls) - 1
            outs = out if isinstance(out, (tuple, list)) else (out,)
            t = next((o for o in outs if isinstance(o, torch.Tensor) and o.requires_grad), None)
            if t is not None:
                t.register_hook(lambda g, c=c, u=u: self._on_call_grad(c, u))
            return None
        return hook

    def _on_call_grad(self, c: int, u: int) -> None:
        """Backward reached call c (its own backward is next): every later call is done."""
        if self._phase != "backward":
            self._phase = "backward"
            self._done_above = len(self._calls)
            self._first_call = {}
            for i, uu in enumerate(self._calls):
                self._first_call.setdefault(uu, i)
        for cc in range(self._done_above - 1, c, -1):
            self._call_done(cc)
        self._done_above = c + 1
        if self.reshard:
            self._prepare_call(c, u)
        return None

    def _prepare_call(self, c: int, u: int) -> None:
        k = c % self.R
        main = self._main if self.fused else None
        if self._gslot_dirty[k]:  # the slot's previous gradients must be reduced everywhere first
            if self._gslot_evt[k] is not None:
                main.wait_event(self._gslot_evt[k])
                self._gslot_evt[k] = None
            self.space.grad[self.slot_base[k]:self.slot_base[k] + self.max_n].zero_()
        self._gslot_dirty[k] = True
        self._bind(u, k)
        if self._slot_unit[k] != u or self._gather_evt[k] is not None:
            if self._gather_evt[k] is not None and self._slot_unit[k] == u:
                main.wait_event(self._gather_evt[k])
            else:
                if self._gather_evt[k] is not None:
                    main.wait_event(self._gather_evt[k])
                self._gather(u, k)
            self._gather_evt[k] = None
            self._slot_unit[k] = u
        if c >= 1 and self.fused:  # next call's unit, on the gather stream, while this call's backward runs
            u2, k2 = self._calls[c - 1], (c - 1) % self.R
            if k2 != k and self._slot_unit[k2] != u2:
                ev = main.record_event()
                self._gs.wait_event(ev)
                self._gs_used = True
                with torch.cuda.stream(self._gs):
                    self._gather(u2, k2)
                self._gather_evt[k2] = self._gs.record_event()
                self._slot_unit[k2] = u2

    def _call_done(self, cc: int) -> None:
        """Call cc's backward is complete on this rank: reduce what it finished."""
        u = self._calls[cc]
        if self.reshard:
            self._reduce_unit(u, cc % self.R, accumulate=u in self._reduced, reuse=True)
            self._reduced.add(u)
            return
        if self._armed and self._first_call.get(u) == cc and not self._unit_reduced[u]:
            self._reduce_unit(u, 0, accumulate=False, reuse=False)

    def _reduce_unit(self, u: int, k: int, accumulate: bool, reuse: bool) -> None:
        """This rank's part of unit u's gradient (slot k) into the fp32 shard gradient."""
        gi = self._gi[u]
        ln, items, blocks = self._blocks[gi]
        self._unit_reduced[u] = True
        if not self.fused:
            a, n, s, _, so = self.layout.groups[gi]
            base = self.slot_base[k] if self.reshard else a
            g = self.space.grad[base:base + n]
            dist.all_reduce(g, group=self.group)
            if ln:
                mine = g[self.rank * s:self.rank * s + ln].float()
                if accumulate:
                    self.gsum[so:so + ln].add_(mine)
                else:
                    self.gsum[so:so + ln].copy_(mine)
            return
        E = ext()
        w, me = self.world, self.rank
        tab, nseg = self._unit_tab[u][k if self.reshard else 0]
        main = self._main
        rs = self._rs if self._rs is not None else main
        if rs is not main:
            rs.wait_event(main.record_event())
            self._rs_used = True
        with torch.cuda.stream(rs):
            E.comm_barrier(self.sig.ptrs, 3, self.epoch_u, True, w, me, self.err)  # every rank done with it
            E.comm_reduce_into(self._grad_buf.ptrs, tab, nseg, items, self.gsum, self.grad_scale(), self.part,
                               self._part_off[gi], blocks, accumulate)
            if reuse:  # every rank has read this slot: it may take the next call's gradients
                E.comm_barrier(self.sig.ptrs, 3, self.epoch_u, True, w, me, self.err)
        if reuse:
            self._gslot_evt[k] = rs.record_event() if rs is not main else None

    def _flush(self) -> None:
        """The backward is over: reduce the calls not reduced yet."""
        if self._phase == "backward":
            for cc in range(self._done_above - 1, -1, -1):
                self._call_done(cc)
            self._done_above = 0
            self._phase = "flushed"

    def _join(self) -> None:
        """The current stream waits for the side streams' work (only streams that
        ran something since the last join: under CUDA-graph capture a stream that
        joined nothing of the capture must not be waited on)."""
        if self.fused:
            cur = torch.cuda.current_stream(self.space.device)
            self._main = cur
            if self._rs is not None and self._rs_used:
                cur.wait_stream(self._rs)
                self._rs_used = False
            if self._gs_used:
                cur.wait_stream(self._gs)
                self._gs_used = False

    # ------------------------------------------------------------ step
    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002
        self.space.zero_grad()
        if self.reshard:
            self._gslot_dirty = [False] * self.R
            for u, k in enumerate(self._bound):  # rebind_grads pointed every unit at slot 0
                if k >= 0:
                    self._bound[u] = -1

    def _update_table(self):
        segs = self.space.active_segments()
        key = tuple(segs)
        if key != self._tab_key:
            upd = self.layout.update_segments(segs, self.rank)
            self._upd = upd
            tab, nseg, items = segment_table([(o, ln) for o, ln, _, _ in upd], self.space.device)
            aux = []
            for so, ln, delta, repl in upd:
                if repl or self.replicate_units:
                    aux += [delta, 1]
                elif self.reshard:
                    aux += [self.S_base, 0]  # this rank's shard store
                else:
                    aux += [delta, 0]
            aux_t = torch.tensor(aux or [0], dtype=torch.long)
            self._tab = (tab, nseg, items, aux_t.to(self.space.device))
            self._tab_key = key
        return self._tab

    @torch.no_grad()
    def step(self, closure=None, hyper: torch.Tensor | None = None, schedule: tuple | None = None):
        loss = closure() if closure is not None else None
        linear_ops.set_prefetch(None)
        self._flush()
        self.step_count += 1
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        tab, nseg, items, aux = self._update_table()
        if self.fused:
            E = ext()
            w, me = self.world, self.rank
            self._join()
            if hyper is not None:
                warm, total, mr = schedule if schedule is not None else (0, 1, 1.0)
                E.adamw_hyper_step(hyper, g.get("initial_lr", lr), b1, b2, warm, total, mr, schedule is not None)
            E.comm_barrier(self.sig.ptrs, 0, self.epoch, True, w, me, self.err)   # all gradients complete
            if self.rep_group is not None:
                ln, it, bl = self._blocks[0]
                E.comm_reduce_into(self._grad_buf.ptrs, self._rep_tab[0], self._rep_tab[1], it, self.gsum,
                                   self.grad_scale(), self.part, 0, bl, False)
            for u in range(len(self.units)):  # units no call reduced (no overlap, or not armed)
                if not self._unit_reduced[u]:
                    gi = self._gi[u]
                    ln, it, bl = self._blocks[gi]
                    E.comm_reduce_into(self._grad_buf.ptrs, self._unit_tab[u][0][0], self._unit_tab[u][0][1], it,
                                       self.gsum, self.grad_scale(), self.part, self._part_off[gi], bl, False)
            E.comm_norm_publish(self.part, self._nparts, self.slots_buf.ptrs, w, me)
            E.comm_barrier(self.sig.ptrs, 1, self.epoch, False, w, me, self.err)  # all shard norms published
            E.comm_adamw_shard(self.gsum, self.master, self.exp_avg, self.exp_avg_sq, self._param_buf.ptrs, 0, w,
                               tab, nseg, items, self.slots_buf.local.view(torch.float32), self.grad_scale(),
                               self.max_grad_norm, lr, b1, b2, eps, wd, self.step_count, self.norm_out, hyper,
                               aux, me)
            E.comm_barrier(self.sig.ptrs, 2, self.epoch, False, w, me, self.err)  # every rank's values written
        else:
            self._step_collective(lr, b1, b2, eps, wd)
        self._after_step()
        return loss

    def _after_step(self) -> None:
        if self.reshard:
            self._slot_unit = [-1] * self.R  # the slots hold last step's values
            self._gather_evt = [None] * self.R
            self._gslot_evt = [None] * self.R
        elif self.world > 1 and not self.replicate_units:
            self.stale = [True] * len(self.units)
        self._reduced = set()
        self._unit_reduced = [False] * len(self.units)
        self._phase = "idle"

    def _step_collective(self, lr, b1, b2, eps, wd):
        s = self.space
        gs = self.grad_scale()
        owned = self.layout.owned(self.rank)
        # the replicated group, and units that no call reduced
        if self.rep_group is not None:
            g = s.grad[:self.n_rep]
            dist.all_reduce(g, group=self.group)
            a, n, sh, _, so = self.rep_group
            ln = self._blocks[0][0]
            if ln:
                self.gsum[so:so + ln].copy_(g[self.rank * sh:self.rank * sh + ln].float())
        for u in range(len(self.units)):
            if not self._unit_reduced[u]:
                self._reduce_unit(u, 0, accumulate=False, reuse=False)
        if s.dtype == torch.float32:
            # fp32 parameters are their own master copy (as in the one-process optimizer), so
            # values a forward wrote into parameter storage (MAC's memory state) are kept
            for fo, so, ln, repl in owned:
                if repl or not self.reshard:
                    self.master[so:so + ln].copy_(s.flat[fo:fo + ln])
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
        self._update_table()
        for so, ln, delta, repl in self._upd:
            gr = self.gsum[so:so + ln] * (gs * coef)
            p, m, v = self.master[so:so + ln], self.exp_avg[so:so + ln], self.exp_avg_sq[so:so + ln]
            p.mul_(1 - lr * wd)
            m.mul_(b1).add_(gr, alpha=1 - b1)
            v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            p.addcdiv_(m, v.sqrt().div_(math.sqrt(bc2)).add_(eps), value=-lr / bc1)
            if self.reshard and not repl:
                self.store[so:so + ln].copy_(p)
            else:
                s.flat[so + delta:so + delta + ln].copy_(p)
        # replicated values (and, for data parallelism, every unit) are all-gathered now
        for a, n, sh, repl, _ in self.layout.groups:
            if repl or self.replicate_units:
                lo = self.rank * sh
                ln = max(0, min(sh, n - lo))
                mine = torch.zeros(sh, dtype=s.flat.dtype, device=s.flat.device)
                if ln:
                    mine[:ln].copy_(s.flat[a + lo:a + lo + ln])
                self._gather_collective(mine, s.flat, a, n, sh)

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
        if self.reshard:  # the gathers' source follows the restored master copy
            for fo, so, ln, repl in self.layout.owned(self.rank):
                if not repl:
                    self.store[so:so + ln].copy_(self.master[so:so + ln])
            self._slot_unit = [-1] * self.R

    def close(self):
        linear_ops.set_prefetch(None)
        for h in self._hooks:
            h.remove()
        self._hooks = []
        for b in self._bufs:
            b.close()


class FullyShardedEngine:
    """Engine for :class:`~titans_pytorch_b200.train.trainer.Trainer` (``engine=``).

    ``reshard=True`` (default) is FSDP's FULL_SHARD: parameters gathered for
    each use and dropped, gradients reduce-scattered during the backward;
    ``reshard=False`` keeps gathered parameters until the step (SHARD_GRAD_OP)."""

    def __init__(self, group=None, reduce: str | None = None, reshard: bool = True, overlap: bool = True,
                 slots: int = 3) -> None:
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
        self.reshard = reshard
        self.overlap = overlap
        self.slots = slots

    def make_optimizer(self, model: nn.Module, cfg):
        fused = self.reduce == "fused" and next(model.parameters()).dtype == torch.bfloat16
        self.reduce = "fused" if fused else "collective"
        return FSDPAdamW(model, cfg, self.group, fused=fused, reshard=self.reshard, overlap=self.overlap,
                         slots=self.slots)

    def reduce_gradients(self, optimizer) -> None:
        """Agree on the set of parameters that received gradients (the reduction
        itself runs during the backward and in the optimizer step)."""
        local = tuple(optimizer.space.got)
        if local != getattr(self, "_last_local", None):
            got = torch.tensor(local, dtype=torch.uint8, device=optimizer.space.device)
            dist.all_reduce(got, op=dist.ReduceOp.MAX, group=self.group)
            self._last_local = local
            self._agreed = [bool(x) for x in got.tolist()]
        optimizer.space.got = list(self._agreed)


ShardedAdamW = FSDPAdamW

__all__ = ["FullyShardedEngine", "FSDPAdamW", "ShardedAdamW", "ShardLayout", "shard_units"]
