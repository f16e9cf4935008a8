"""``OptimizedTrainer`` / ``OptimizedTrainingConfig`` API (`src/titans/optimized_training.py:50-457`).

The reference's optimized trainer adds autocast + GradScaler, torch.compile and
CUDA-graph capture around a plain step.  Here the step is already the fused
bf16 path of :class:`Trainer` (fp32 master weights, device-side clip and
AdamW), so this class maps the reference's configuration onto it:

* ``mixed_precision`` selects the compute dtype (bf16 or fp32; fp16 is
  refused -- the kernels compute in bf16);
* ``gradient_checkpointing`` enables block recomputation;
* ``use_cuda_graphs`` -- and ``use_compile``, whose reduce-overhead mode is
  the same thing -- capture the whole step (forward, backward, clip, AdamW)
  in a CUDA graph and replay it (CUDA device, no gradient accumulation);
* ``profile_enabled`` records the first ``profile_steps`` steps with the
  PyTorch profiler and keeps a per-kernel table (own kernels / libraries /
  ATen) in ``profile_summary`` (the reference's `optimized_training.py:535-561`
  only times a region).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops.attention import NO_WINDOW, window_attention
from ..utils.perf import enable_gradient_checkpointing
from .trainer import Trainer, TrainStepConfig


@dataclass
class OptimizedTrainingConfig:
    learning_rate: float = 4e-4
    weight_decay: float = 0.1
    betas: tuple[float, float] = (0.9, 0.95)
    max_grad_norm: float = 1.0
    gradient_accumulation_steps: int = 1
    mixed_precision: str = "bf16"        # "bf16" | "fp32"
    use_compile: bool = False
    use_cuda_graphs: bool = False
    gradient_checkpointing: bool = False
    warmup_steps: int = 0
    total_steps: int = 0
    profile_enabled: bool = False
    profile_steps: int = 0


class OptimizedTrainer:
    def __init__(self, model: torch.nn.Module, config: OptimizedTrainingConfig | None = None, device=None,
                 engine=None) -> None:
        self.config = c = config or OptimizedTrainingConfig()
        if c.mixed_precision in ("fp16", "float16"):
            raise ValueError("fp16 is not supported: the sm_100a kernels compute in bf16 (use bf16 or fp32)")
        dtype = torch.bfloat16 if c.mixed_precision in ("bf16", "bfloat16") else torch.float32
        if c.gradient_checkpointing:
            enable_gradient_checkpointing(model)
        if device is None:
            device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        graph = ((c.use_cuda_graphs or c.use_compile) and torch.device(device).type == "cuda"
                 and c.gradient_accumulation_steps == 1)
        self.trainer = Trainer(model, TrainStepConfig(
            lr=c.learning_rate, weight_decay=c.weight_decay, betas=c.betas, grad_clip=c.max_grad_norm,
            warmup_steps=c.warmup_steps, total_steps=c.total_steps,
            gradient_accumulation_steps=c.gradient_accumulation_steps, dtype=dtype, cuda_graph=graph),
            device=device, engine=engine)
        self.uses_cuda_graph = graph
        self.model = self.trainer.model
        self.optimizer = self.trainer.optimizer
        self.profile_summary: dict | None = None
        self._prof = None
        self._prof_left = c.profile_steps if c.profile_enabled else 0

    @property
    def global_step(self) -> int:
        return self.trainer.global_step

    def _step(self, batch) -> torch.Tensor:
        if self._prof_left > 0 and self._prof is None:
            from torch.profiler import ProfilerActivity, profile

            acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
            self._prof = profile(activities=acts)
            self._prof.__enter__()
        loss = self.trainer.train_step(batch)
        if self._prof is not None:
            self._prof_left -= 1
            if self._prof_left <= 0:
                if torch.cuda.is_available():
                    torch.cuda.synchronize()
                self._prof.__exit__(None, None, None)
                self.profile_summary = _kernel_table(self._prof, self.config.profile_steps)
                self._prof = None
        return loss

    def train_step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return self._step({"input_ids": input_ids, "labels": labels})

    def train_epoch(self, loader, log_every: int = 0, sink=print) -> float:
        total, n = None, 0
        for i, batch in enumerate(loader):
            loss = self._step(batch)
            total = loss if total is None else total + loss
            n += 1
            if log_every and (i + 1) % log_every == 0:
                sink(f"step {self.global_step} loss {float(loss):.4f}")
        return float(total / max(n, 1)) if total is not None else float("nan")


def _kernel_table(prof, steps: int) -> dict:
    """Device time per kernel class and the top kernels of a profiled run (ms per step)."""
    import collections

    from ..cli.step_profile import classify

    per_class, per_kernel = collections.Counter(), collections.Counter()
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        us = e.device_time if hasattr(e, "device_time") else e.cuda_time
        c = "copy" if ("memcpy" in e.name.lower() or "memset" in e.name.lower()) else classify(e.name)
        per_class[c] += us
        per_kernel[(c, e.name)] += us
    n = max(1, steps)
    return {"classes_ms_per_step": {c: v / 1000 / n for c, v in per_class.items()},
            "top": [(c, k[:120], v / 1000 / n) for (c, k), v in per_kernel.most_common(15)]}


def memory_efficient_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                               window: int | None = None, scale: float | None = None) -> torch.Tensor:
    """Causal (optionally windowed) attention of q/k/v [B, H, T, d] without a T x T mask.

    Runs the framework's flash kernels (no RoPE); returns [B, H, T, d].
    """
    if not causal:
        raise NotImplementedError("only causal attention is provided")
    B, H, T, d = q.shape
    qkv = torch.cat([t.transpose(1, 2).reshape(B, T, H * d) for t in (q, k, v)], dim=-1)
    o = window_attention(qkv, None, H, window=window if window is not None else NO_WINDOW, scale=scale)
    return o.transpose(1, 2)
