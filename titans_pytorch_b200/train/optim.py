"""Flat-buffer AdamW with the global-norm clip inside the update.

The reference trains with ``torch.optim.AdamW(fused=True, betas=(0.9, 0.95))``
and ``clip_grad_norm_`` (`scripts/pretrain.py:506-519, 607-625`).  Here:

* every trainable parameter becomes a view into ONE flat buffer (the model's
  compute dtype, e.g. bf16), and its ``.grad`` a view into one flat gradient
  buffer, so autograd accumulates straight into it;
* the optimizer keeps fp32 master weights and fp32 moments for the flat range;
* one kernel computes the global gradient norm and the clip coefficient on the
  device, a second applies AdamW to every parameter that received a gradient
  this step and writes the new compute-dtype weights -- no host sync.

Parameters that got no gradient in a step are skipped entirely (no weight
decay, no moment decay), which is what ``torch.optim.AdamW`` does for
``grad is None``; a post-accumulate hook records which ones did.

The data-parallel engine (:mod:`titans_pytorch_b200.parallel.ddp`) subclasses
this with the gradient reduction fused into the same update.
"""

from __future__ import annotations

import math

import torch

from ..ops._ext import ext, want_kernels

ALIGN = 64  # elements; keeps every parameter view 128-byte aligned for bf16


def unique_trainable(params) -> list:
    """Trainable parameters in order, each once (tied weights appear once)."""
    seen, plist = set(), []
    for p in params:
        if p.requires_grad and id(p) not in seen:
            seen.add(id(p))
            plist.append(p)
    if not plist:
        raise ValueError("no trainable parameters")
    return plist


def intersect_segments(segs, lo: int, hi: int) -> list[tuple[int, int]]:
    """Active (offset, length) ranges clipped to [lo, hi), made relative to lo."""
    out = []
    for o, n in segs:
        a, b = max(o, lo), min(o + n, hi)
        if a < b:
            out.append((a - lo, b - a))
    return out


class FlatParamSpace:
    """Owns the flat parameter and gradient buffers of a set of parameters."""

    def __init__(self, params, grad_dtype: torch.dtype | None = None, pad_to: int = 1,
                 buffers=None, placement=None) -> None:
        """``pad_to``: round the total length up to a multiple of it (e.g. ALIGN*world for
        sharding).  ``buffers``: optional callable ``(total, dtype) -> (flat, grad)`` that
        provides the two flat buffers (e.g. peer-visible memory); zero-filled.

        ``placement``: optional ``(phys, total)``: parameter i lives at ``phys[i]`` of
        buffers of ``total`` elements instead of its logical offset (parameters may
        share memory, e.g. the working slots of a sharded-parameter engine; their
        values are then not copied in).  ``offsets`` stay logical (optimizer
        bookkeeping, ``active_segments``); ``phys`` is where the views point."""
        plist = unique_trainable(params)
        self.params = plist
        self.device = plist[0].device
        self.dtype = plist[0].dtype
        if any(p.dtype != self.dtype or p.device != self.device for p in plist):
            raise ValueError("all parameters must share dtype and device")
        self.offsets, off = [], 0
        for p in plist:
            self.offsets.append(off)
            off += (p.numel() + ALIGN - 1) // ALIGN * ALIGN
        self.logical_total = off
        if placement is None:
            self.phys = list(self.offsets)
            self.total = (off + pad_to - 1) // pad_to * pad_to
            copy_in = [True] * len(plist)
        else:
            self.phys, self.total = list(placement[0]), int(placement[1])
            counts: dict[int, int] = {}
            for o in self.phys:
                counts[o] = counts.get(o, 0) + 1
            copy_in = [counts[o] == 1 for o in self.phys]
        if buffers is not None:
            self.flat, self.grad = buffers(self.total, self.dtype)
        else:
            self.flat = torch.zeros(self.total, dtype=self.dtype, device=self.device)
            self.grad = torch.zeros(self.total, dtype=grad_dtype or self.dtype, device=self.device)
        with torch.no_grad():
            for p, o, cp in zip(plist, self.phys, copy_in, strict=True):
                n = p.numel()
                if cp:
                    self.flat[o:o + n].copy_(p.detach().reshape(-1))
                p.data = self.flat[o:o + n].view_as(p)
                p.grad = self.grad[o:o + n].view_as(p)
        self.got = [False] * len(plist)
        self._hooks = [p.register_post_accumulate_grad_hook(self._make_hook(i))
                       for i, p in enumerate(plist)]
        for i, p in enumerate(plist):  # for gradients written in place (ops.linear)
            p._titans_grad_mark = self._make_hook(i)

    def _make_hook(self, i):
        def hook(_p):
            self.got[i] = True
        return hook

    def rebind_grads(self) -> None:
        """Re-attach the flat gradient views (after a caller set .grad = None)."""
        for p, o in zip(self.params, self.phys):
            if p.grad is None or p.grad.data_ptr() != self.grad[o:o + 1].data_ptr():
                p.grad = self.grad[o:o + p.numel()].view_as(p)

    def zero_grad(self) -> None:
        self.rebind_grads()
        self.grad.zero_()
        self.got = [False] * len(self.params)

    def active_segments(self) -> list[tuple[int, int]]:
        """Merged (offset, length) ranges of parameters that received a gradient."""
        segs: list[list[int]] = []
        for i, (p, o) in enumerate(zip(self.params, self.offsets)):
            if not self.got[i]:
                continue
            n = (p.numel() + ALIGN - 1) // ALIGN * ALIGN
            if segs and segs[-1][0] + segs[-1][1] == o:
                segs[-1][1] += n
            else:
                segs.append([o, n])
        return [(a, b) for a, b in segs]


def segment_table(segs: list[tuple[int, int]], device, chunk: int = 1 << 14):
    """Device table consumed by the optimizer kernels: offsets, lengths, item starts."""
    n = len(segs)
    if any(o % 8 or ln % 8 for o, ln in segs):
        raise ValueError("optimizer segments must be 8-element aligned (the kernels move 8 elements per access)")
    tab = torch.empty(3 * n, dtype=torch.long)
    items = 0
    for i, (o, ln) in enumerate(segs):
        tab[2 * i], tab[2 * i + 1], tab[2 * n + i] = o, ln, items
        items += (ln + chunk - 1) // chunk
    return tab.to(device), n, items


class FusedAdamW(torch.optim.Optimizer):
    """AdamW over a :class:`FlatParamSpace` with an optional in-kernel global-norm clip."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, max_grad_norm: float = 0.0,
                 use_kernels: bool | None = None) -> None:
        self.space = params if isinstance(params, FlatParamSpace) else FlatParamSpace(params)
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)
        super().__init__(self.space.params, defaults)
        s = self.space
        self.max_grad_norm = float(max_grad_norm)
        self.kernels = want_kernels(s.flat, use_kernels)
        self.master = s.flat if s.dtype == torch.float32 else s.flat.float()
        self.exp_avg = torch.zeros(s.total, dtype=torch.float32, device=s.device)
        self.exp_avg_sq = torch.zeros(s.total, dtype=torch.float32, device=s.device)
        self.step_count = 0
        self._tab_key = None
        self._tab = None
        self.last_grad_norm: torch.Tensor | None = None
        self.graph_safe = self.kernels  # the step can be captured in a CUDA graph

    # torch.optim API -----------------------------------------------------
    def zero_grad(self, set_to_none: bool = True) -> None:  # noqa: ARG002 (flat grads are reused)
        self.space.zero_grad()

    def _table(self):
        segs = self.space.active_segments()
        key = tuple(segs)
        if key != self._tab_key:
            self._tab = segment_table(segs, self.space.device)
            self._tab_key = key
        return self._tab

    def grad_scale(self) -> float:
        """Multiplier applied to the raw flat gradient (1 here; 1/world in DP)."""
        return 1.0

    def make_hyper(self) -> torch.Tensor:
        """Device copy of the step-dependent values for CUDA-graph replay:
        ``[step, lr, 1 - b1^step, sqrt(1 - b2^step)]``, starting at this step."""
        return torch.tensor([float(self.step_count), 0.0, 0.0, 0.0], dtype=torch.float32, device=self.space.device)

    @torch.no_grad()
    def step(self, closure=None, hyper: torch.Tensor | None = None, schedule: tuple | None = None):
        """One update.  With ``hyper`` (see :meth:`make_hyper`) the step count,
        learning rate and bias corrections are advanced and read on the device
        (``schedule`` = (warmup, total, min_ratio) or None), so the launch
        sequence is identical every step and can be replayed from a CUDA graph."""
        loss = closure() if closure is not None else None
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        self.step_count += 1
        s = self.space
        tab, nseg, items = self._table()
        gs = self.grad_scale()
        if self.kernels:
            E = ext()
            clip = None
            if self.max_grad_norm > 0:
                clip = E.grad_norm_clip(s.grad, tab, nseg, items, gs, self.max_grad_norm)
                self.last_grad_norm = clip[0]
            out = None if self.master is s.flat else s.flat
            if hyper is not None:
                base = g.get("initial_lr", lr)
                warm, total, mr = schedule if schedule is not None else (0, 1, 1.0)
                E.adamw_hyper_step(hyper, base, b1, b2, warm, total, mr, schedule is not None)
            E.adamw_step(self.master, self.exp_avg, self.exp_avg_sq, s.grad, out, tab, nseg, items,
                         clip, gs, lr, b1, b2, eps, wd, self.step_count, hyper)
        else:
            self._step_reference(lr, b1, b2, eps, wd, gs)
        return loss

    def _step_reference(self, lr, b1, b2, eps, wd, gs):
        s = self.space
        segs = s.active_segments()
        coef = 1.0
        if self.max_grad_norm > 0:
            tot = sum(float((s.grad[o:o + n].float() * gs).pow(2).sum()) for o, n in segs)
            nrm = math.sqrt(tot)
            self.last_grad_norm = torch.tensor(nrm)
            coef = min(1.0, self.max_grad_norm / (nrm + 1e-6))
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        for o, n in segs:
            gr = s.grad[o:o + n].float() * (gs * coef)
            p = self.master[o:o + n]
            m = self.exp_avg[o:o + n]
            v = self.exp_avg_sq[o:o + n]
            p.mul_(1 - lr * wd)
            m.mul_(b1).add_(gr, alpha=1 - b1)
            v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
            p.addcdiv_(m, v.sqrt().div_(math.sqrt(bc2)).add_(eps), value=-lr / bc1)
            if self.master is not s.flat:
                s.flat[o:o + n].copy_(p)

    # checkpointing ---------------------------------------------------------
    def state_dict(self):
        return {"step": self.step_count, "master": self.master, "exp_avg": self.exp_avg,
                "exp_avg_sq": self.exp_avg_sq, "param_groups": [
                    {k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, sd):
        self.step_count = int(sd["step"])
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for g, sg in zip(self.param_groups, sd["param_groups"]):
            g.update(sg)
        if self.master is not self.space.flat:
            self.space.flat.copy_(self.master)
