"""Pipeline parallelism for MAC: the (layer, segment) wavefront across ranks.

The reference runs MAC's segments through all layers one at a time
(`src/titans/models.py:301-314`).  Block i on segment c depends on block i-1
on segment c and on block i's memory state after segment c-1 only, so with
the layers split into contiguous stages, one per rank, segment c can be in
stage s while segment c+1 is in stage s-1: a pipeline whose micro-batches
are the segments.

* Forward: stage 0 embeds each segment; every stage runs its blocks on the
  segment (its memory states carried from the previous segment) and sends the
  output to the next stage without waiting (point-to-point: NCCL over NVLink
  on GPUs, gloo on CPU).  The last stage applies the final norm, the tied head
  and the loss.
* Backward, per segment in reverse order: the memory states are detached
  between segments (the reference's `memory.py:461`), so the segments'
  autograd graphs are independent; the last stage back-propagates segment c's
  share of the mean loss and sends the gradient of its input back while it
  starts on segment c-1, and every stage does the same with the gradient it
  receives.
* The embedding and the head share one weight: its gradient is summed between
  the first and the last stage.  The global gradient norm for clipping is
  reduced over the stages.

Every rank holds the whole model (checkpoints are the unsharded format) and
computes only its stage; :meth:`MACPipeline.parameters` lists what it trains.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops.linear import linear
from ..ops.loss import cross_entropy


def split_layers(num_layers: int, stages: int) -> list[tuple[int, int]]:
    """Contiguous, balanced ``[lo, hi)`` layer ranges, one per stage."""
    if stages > num_layers:
        raise ValueError(f"{stages} pipeline stages need at least as many layers (got {num_layers})")
    base, extra = divmod(num_layers, stages)
    out, lo = [], 0
    for s in range(stages):
        hi = lo + base + (1 if s < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


class MACPipeline:
    """One rank's stage of a pipeline-parallel TitansMAC."""

    def __init__(self, model, group=None) -> None:
        if getattr(model, "model_type", None) != "mac":
            raise NotImplementedError("the segment pipeline is for MAC models")
        self.model, self.group = model, group
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        self.lo, self.hi = split_layers(len(model.blocks), self.world)[self.rank]
        self.first, self.last = self.rank == 0, self.rank == self.world - 1
        g = (lambda r: r) if group is None else (lambda r: dist.get_global_rank(group, r))
        self.prev = g(self.rank - 1) if not self.first else None
        self.next = g(self.rank + 1) if not self.last else None

    def parameters(self) -> list:
        """The parameters this stage computes gradients for and updates."""
        m = self.model
        ps = [p for b in m.blocks[self.lo:self.hi] for p in b.parameters()]
        if self.first or self.last:
            ps.append(m.embed.weight)  # tied with the head
        if self.last:
            ps += list(m.norm.parameters())
        return [p for p in dict.fromkeys(ps) if p.requires_grad]

    def _segments(self, T: int):
        cs = self.model.config.chunk_size
        return [(s, min(cs, T - s)) for s in range(0, T, cs)]

    def forward_backward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None, states=None,
                         loss_scale: float = 1.0, sync_tied: bool = True):
        """One pipelined forward (and, with ``labels``, backward) of a batch.

        Every rank passes the same ``input_ids`` (stage 0 embeds them) and
        ``labels`` (the last stage's loss).  Returns ``(loss, states)``: the mean
        loss on every rank (a detached scalar) and this stage's new memory
        states.  ``loss_scale`` scales the back-propagated loss (gradient
        accumulation), not the returned value.  ``sync_tied=False`` leaves the
        tied weight's gradient unsummed (call :meth:`sync_tied_grads` once after
        the last accumulated micro-batch).
        """
        m = self.model
        blocks = m.blocks[self.lo:self.hi]
        states = list(states) if states is not None else [None] * len(blocks)
        B, T = input_ids.shape
        D = m.config.dim
        dev, dt = m.embed.weight.device, m.embed.weight.dtype
        train = labels is not None and torch.is_grad_enabled()
        segs = self._segments(T)
        ins, outs, pending = [], [], []
        for s, n in segs:
            if self.first:
                x = m.embed(input_ids[:, s:s + n])
            else:
                x = torch.empty(B, n, D, device=dev, dtype=dt)
                dist.recv(x, src=self.prev, group=self.group)
                x.requires_grad_(train)
            ins.append(x)
            for j, blk in enumerate(blocks):
                x, states[j] = blk(x, state=states[j])
            outs.append(x)
            if not self.last:
                t = x.detach().contiguous()
                pending.append((dist.isend(t, dst=self.next, group=self.group), t))
        for w, _ in pending:
            w.wait()
        if labels is not None:
            total = (labels != -100).sum().clamp_min(1).to(torch.float32)
        loss = torch.zeros((), device=dev, dtype=torch.float32)
        if self.last:
            uk = getattr(m.config, "use_kernels", None)
            for c in range(len(segs) - 1, -1, -1):
                s, n = segs[c]
                if labels is None:
                    continue
                lab = labels[:, s:s + n]
                cnt = (lab != -100).sum().to(torch.float32)
                part = cross_entropy(linear(m.norm(outs[c]), m.head.weight, use_kernels=uk), lab,
                                     use_kernels=uk) * (cnt / total)
                if train:
                    (part * loss_scale if loss_scale != 1.0 else part).backward()
                    if not self.first:
                        self._send_grad(ins[c])
                loss += part.detach().float()
        elif train:
            for c in range(len(segs) - 1, -1, -1):
                g = torch.empty_like(outs[c])
                dist.recv(g, src=self.next, group=self.group)
                torch.autograd.backward(outs[c], g)
                if not self.first:
                    self._send_grad(ins[c])
        if labels is not None and self.world > 1:
            dist.broadcast(loss, src=self.world - 1 if self.group is None else dist.get_global_rank(
                self.group, self.world - 1), group=self.group)
        if train and sync_tied:
            self.sync_tied_grads()
        return loss, states

    def make_optimizer(self, lr: float = 4e-4, betas=(0.9, 0.95), weight_decay: float = 0.1):
        """AdamW over this stage's parameters (the clip is done across stages by
        :meth:`train_step`, so the optimizer does not clip)."""
        from ..train.optim import FusedAdamW

        return FusedAdamW(self.parameters(), lr=lr, betas=betas, weight_decay=weight_decay, max_grad_norm=0.0,
                          use_kernels=getattr(self.model.config, "use_kernels", None))

    def train_step(self, batch: dict, optimizer, max_grad_norm: float = 1.0) -> torch.Tensor:
        """Forward, backward, cross-stage clip and this stage's AdamW step."""
        dev = self.model.embed.weight.device
        ids = batch["input_ids"].to(dev, non_blocking=True)
        labels = batch["labels"].to(dev, non_blocking=True)
        loss, _ = self.forward_backward(ids, labels)
        if max_grad_norm > 0:
            self.clip_grad_norm_(max_grad_norm)
        optimizer.step()
        optimizer.zero_grad()
        return loss

    def sync_parameters(self) -> None:
        """Bring every rank's copy of every stage's parameters up to date (each
        stage's owner broadcasts them), e.g. before a checkpoint is written."""
        if self.world == 1:
            return
        m = self.model
        g = (lambda r: r) if self.group is None else (lambda r: dist.get_global_rank(self.group, r))
        with torch.no_grad():
            for s, (lo, hi) in enumerate(split_layers(len(m.blocks), self.world)):
                for p in (q for b in m.blocks[lo:hi] for q in b.parameters()):
                    dist.broadcast(p.data, src=g(s), group=self.group)
            for p in m.norm.parameters():
                dist.broadcast(p.data, src=g(self.world - 1), group=self.group)
            dist.broadcast(m.embed.weight.data, src=g(0), group=self.group)

    def _send_grad(self, x: torch.Tensor) -> None:
        g = x.grad if x.grad is not None else torch.zeros_like(x)
        dist.send(g.contiguous(), dst=self.prev, group=self.group)

    def sync_tied_grads(self) -> None:
        """Sum the embedding / head weight's gradient over the first and last stage."""
        if self.world == 1:
            return
        w = self.model.embed.weight
        g = w.grad if (w.grad is not None and (self.first or self.last)) else torch.zeros_like(w)
        g = g.contiguous()
        dist.all_reduce(g, group=self.group)
        if self.first or self.last:
            if w.grad is None:
                w.grad = g
            else:
                w.grad.copy_(g)

    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        """Global-norm clip over all stages (the tied weight counted once)."""
        params = self.parameters()
        sq = torch.zeros((), device=self.model.embed.weight.device, dtype=torch.float32)
        for p in params:
            if p.grad is None or (p is self.model.embed.weight and not self.first):
                continue
            sq += p.grad.float().pow(2).sum()
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        norm = sq.sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
        for p in params:
            if p.grad is not None:
                p.grad.mul_(coef.to(p.grad.dtype))
        return norm


class PipelineEngine:
    """Training engine for :class:`~titans_pytorch_b200.train.trainer.Trainer`
    that runs a MAC model as a pipeline over the ranks of ``group``: the
    trainer hands it each batch (the same batch on every rank), it runs the
    pipelined forward and backward, clips over the stages and steps this
    stage's AdamW.  Checkpoints gather every stage's parameters into the
    unsharded model file and keep one optimizer file per stage."""

    graph_safe = False

    def __init__(self, group=None) -> None:
        self.group = group
        self.pipe: MACPipeline | None = None
        self.clip = 0.0

    def make_optimizer(self, model, cfg):
        from ..train.optim import FusedAdamW

        self.pipe = MACPipeline(model, self.group)
        self.clip = float(cfg.grad_clip)
        opt = FusedAdamW(self.pipe.parameters(), lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                         weight_decay=cfg.weight_decay, max_grad_norm=0.0,
                         use_kernels=getattr(model.config, "use_kernels", None))
        opt.shard_state = self.pipe.world > 1  # one optimizer file per stage

        def full_model_state_dict(m):
            self.pipe.sync_parameters()
            return m.state_dict()

        opt.full_model_state_dict = full_model_state_dict
        return opt

    def forward_backward(self, input_ids, labels, loss_scale: float = 1.0) -> torch.Tensor:
        # the tied weight's gradient is summed once per optimizer step, in reduce_gradients
        return self.pipe.forward_backward(input_ids, labels, loss_scale=loss_scale, sync_tied=False)[0]

    def reduce_gradients(self, optimizer) -> None:
        self.pipe.sync_tied_grads()
        if self.clip > 0:
            self.pipe.clip_grad_norm_(self.clip)


__all__ = ["MACPipeline", "PipelineEngine", "split_layers"]
