"""Training step / loop for Titans models.

Mirrors the reference trainer's step (`scripts/pretrain.py:559-625`): forward,
mean token cross-entropy, backward, global-norm clip, AdamW(beta=(0.9, 0.95)),
LR schedule (linear warm-up then cosine to a 0.1 floor, `:408-425`).  The
differences are the B200 ones: the model computes in bf16 with fp32 master
weights held by :class:`FusedAdamW`; clip and update are device kernels; the
loss stays on the device until the caller asks for it; with a process group,
gradients are reduced by the data-parallel engine before the update.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops.linear import accumulate_weight_grads
from ..ops.loss import cross_entropy
from .optim import FusedAdamW


def cosine_with_warmup(step: int, warmup: int, total: int, min_ratio: float = 0.1) -> float:
    """LR multiplier: linear warm-up, then cosine decay to ``min_ratio``."""
    if step < warmup:
        return float(step) / float(max(1, warmup))
    progress = float(step - warmup) / float(max(1, total - warmup))
    return max(min_ratio, 0.5 * (1.0 + math.cos(math.pi * progress)))


def get_cosine_schedule_with_warmup(optimizer, num_warmup_steps: int, num_training_steps: int,
                                    min_lr_ratio: float = 0.1):
    return torch.optim.lr_scheduler.LambdaLR(
        optimizer, lambda s: cosine_with_warmup(s, num_warmup_steps, num_training_steps, min_lr_ratio))


@dataclass
class TrainStepConfig:
    lr: float = 4e-4
    weight_decay: float = 0.1
    betas: tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    grad_clip: float = 1.0
    warmup_steps: int = 0
    total_steps: int = 0          # 0: constant LR after warm-up
    min_lr_ratio: float = 0.1
    gradient_accumulation_steps: int = 1
    dtype: torch.dtype = torch.bfloat16
    # Capture the whole step (forward, backward, clip, AdamW, zero-grad) in a
    # CUDA graph after `graph_warmup` eager steps and replay it afterwards.
    cuda_graph: bool = False
    graph_warmup: int = 3


class Trainer:
    """One-GPU (or data-parallel, see ``engine``) training driver."""

    def __init__(self, model: torch.nn.Module, cfg: TrainStepConfig | None = None,
                 device: torch.device | str | None = None, engine=None) -> None:
        self.cfg = cfg or TrainStepConfig()
        if device is None:
            device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        self.device = torch.device(device)
        self.model = model.to(device=self.device, dtype=self.cfg.dtype)
        self.engine = engine
        if engine is not None:
            self.optimizer = engine.make_optimizer(self.model, self.cfg)
        else:
            self.optimizer = FusedAdamW(self.model.parameters(), lr=self.cfg.lr, betas=self.cfg.betas,
                                        eps=self.cfg.eps, weight_decay=self.cfg.weight_decay,
                                        max_grad_norm=self.cfg.grad_clip,
                                        use_kernels=getattr(self.model.config, "use_kernels", None))
        self.scheduler = None
        if self.cfg.total_steps > 0 or self.cfg.warmup_steps > 0:
            self.scheduler = get_cosine_schedule_with_warmup(
                self.optimizer, self.cfg.warmup_steps, max(self.cfg.total_steps, 1), self.cfg.min_lr_ratio)
        self.global_step = 0
        self._micro = 0
        self.optimizer.zero_grad()
        # small weight gradients on a second stream, unless the engine reads the
        # gradients during the backward (reductions of finished blocks)
        self._side_wgrad = self.device.type == "cuda" and not getattr(self.optimizer, "reduces_during_backward", False)
        if getattr(self.model, "wavefront_streams", 0) > 1 and getattr(self.optimizer, "reduces_during_backward",
                                                                        False):
            raise ValueError("the MAC wavefront runs the backward on several streams; use an engine that "
                             "reduces the gradients after the backward")
        self._graph = None
        self._eager_graph_steps = 0
        if self.cfg.cuda_graph:
            if self.device.type != "cuda" or self.cfg.gradient_accumulation_steps != 1:
                raise ValueError("cuda_graph needs a CUDA device and no gradient accumulation")
            if any(getattr(getattr(b, "cp", None), "active", False) for b in getattr(self.model, "blocks", ())):
                raise ValueError("cuda_graph does not capture context parallelism (its halo exchange and "
                                 "memory all-reduce are host-issued point-to-point calls)")
            if getattr(engine, "forward_backward", None) is not None:
                raise ValueError("cuda_graph does not capture an engine that runs its own forward and "
                                 "backward (pipeline stages)")
            if not getattr(self.optimizer, "graph_safe", False):
                raise ValueError("cuda_graph needs a graph-safe optimizer (fused kernels; the fused "
                                 "data-parallel engine, not the collective one)")

    def _to_device(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(self.device, non_blocking=True)

    def loss_fn(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        logits, _ = self.model(input_ids)
        return cross_entropy(logits, labels, use_kernels=getattr(self.model.config, "use_kernels", None))

    def train_step(self, batch: dict[str, torch.Tensor]) -> torch.Tensor:
        """Forward + backward (+ optimizer step at accumulation boundaries).

        ``batch`` holds ``input_ids`` and ``labels`` (host or device tensors).
        Returns the micro-batch loss as a device tensor (no host sync).
        """
        self.model.train()
        if self.cfg.cuda_graph:
            return self._graph_step(batch)
        ids = self._to_device(batch["input_ids"])
        labels = self._to_device(batch["labels"])
        accum = self.cfg.gradient_accumulation_steps
        fb = getattr(self.engine, "forward_backward", None)
        if fb is not None:  # an engine that runs the forward and backward itself (pipeline stages)
            loss = fb(ids, labels, loss_scale=1.0 / accum)
        else:
            loss = self.loss_fn(ids, labels)
            prep = getattr(self.optimizer, "prepare_backward", None)
            if prep is not None:  # engines that reduce during the backward: is this the step's last one?
                prep((self._micro + 1) % accum == 0)
            self._backward(loss / accum if accum > 1 else loss)
        self._micro += 1
        if self._micro % accum == 0:
            self.optimizer_step()
        return loss.detach()

    def _backward(self, loss: torch.Tensor) -> None:
        with accumulate_weight_grads(side_stream=self._side_wgrad):
            loss.backward()
            join = getattr(self.model, "join_streams", None)
            if join is not None:  # a model whose forward (so its backward) used several streams
                join()

    # ------------------------------------------------------------ CUDA graph
    def _schedule(self):
        if self.scheduler is None:
            return None
        return (self.cfg.warmup_steps, max(self.cfg.total_steps, 1), self.cfg.min_lr_ratio)

    def _graph_step(self, batch) -> torch.Tensor:
        """Eager warm-up steps on a side stream, then one capture, then replays.

        Every replay runs the same kernels on the same buffers: the batch is
        copied into static input tensors, and the step count, learning rate and
        bias corrections live on the device (see ``FusedAdamW.step``).
        """
        cur = torch.cuda.current_stream(self.device)
        if self._graph is None and self._eager_graph_steps < self.cfg.graph_warmup:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                ids = self._to_device(batch["input_ids"])
                labels = self._to_device(batch["labels"])
                loss = self.loss_fn(ids, labels)
                self._backward(loss)
                self.optimizer_step()
            cur.wait_stream(side)
            self._eager_graph_steps += 1
            return loss.detach()
        if self._graph is None:
            self._capture(batch)
        self._static_ids.copy_(batch["input_ids"], non_blocking=True)
        self._static_labels.copy_(batch["labels"], non_blocking=True)
        self._graph.replay()
        self.optimizer.step_count += 1
        self.global_step += 1
        return self._static_loss

    def _capture(self, batch) -> None:
        self._static_ids = batch["input_ids"].to(self.device).clone()
        self._static_labels = batch["labels"].to(self.device).clone()
        self._hyper = self.optimizer.make_hyper()
        sched = self._schedule()
        opt = self.optimizer
        opt.zero_grad()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        saved_count = opt.step_count
        with torch.cuda.graph(g):
            loss = self.loss_fn(self._static_ids, self._static_labels)
            self._backward(loss)
            if self.engine is not None:
                self.engine.reduce_gradients(opt)
            opt.step(hyper=self._hyper, schedule=sched)
            opt.zero_grad()
            self._static_loss = loss.detach()
        opt.step_count = saved_count  # capture recorded the work without running it
        self._graph = g

    def optimizer_step(self) -> None:
        if self.engine is not None:
            self.engine.reduce_gradients(self.optimizer)
        self.optimizer.step()
        if self.scheduler is not None:
            self.scheduler.step()
        self.optimizer.zero_grad()
        self.global_step += 1

    @torch.no_grad()
    def evaluate(self, batches, group=None, max_batches: int | None = None) -> dict[str, float]:
        """Mean token loss over ``batches`` (and, in a process group, over every
        rank's batches: the (loss sum, token count) pair is all-reduced, as the
        reference gathers its eval losses, `scripts/pretrain_distributed.py:479-518`).
        Sums stay on the device until the end (one host read)."""
        import torch.distributed as dist

        self.model.eval()
        acc = torch.zeros(2, dtype=torch.float64, device=self.device)
        for i, b in enumerate(batches):
            if max_batches is not None and i >= max_batches:
                break
            ids = self._to_device(b["input_ids"])
            labels = self._to_device(b["labels"])
            fb = getattr(self.engine, "forward_backward", None)
            if fb is not None:  # pipeline stages: the pipelined forward's loss (same on every rank)
                loss = fb(ids, labels)
            else:
                logits, _ = self.model(ids)
                loss = cross_entropy(logits, labels, use_kernels=getattr(self.model.config, "use_kernels", None))
            k = (labels != -100).sum()
            acc[0] += loss.double() * k
            acc[1] += k
        self.model.train()
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(acc, group=group)
        tot, n = acc.tolist()
        avg = tot / max(n, 1.0)
        return {"val_loss": avg, "val_ppl": math.exp(min(avg, 20.0)), "val_tokens": int(n)}

    def check_errors(self) -> None:
        """Raise if a bounded device wait of this trainer's kernels ran out
        (see :mod:`titans_pytorch_b200.parallel.health`); synchronises."""
        from ..parallel.health import check_device_errors

        check_device_errors(self.optimizer, self.device if self.device.type == "cuda" else None)
