"""``OptimizedTrainer`` / ``OptimizedTrainingConfig`` API (`src/titans/optimized_training.py:50-457`).

The reference's optimized trainer adds autocast + GradScaler, torch.compile and
CUDA-graph capture around a plain step.  Here the step is already the fused
bf16 path of :class:`Trainer` (fp32 master weights, device-side clip and
AdamW), so this class maps the reference's configuration onto it:
``mixed_precision`` selects the compute dtype, ``gradient_checkpointing``
enables block recomputation, ``use_compile``/``use_cuda_graphs`` are accepted
and ignored for training (the hot path is native kernels, not a compiler).
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
        dtype = torch.bfloat16 if c.mixed_precision in ("bf16", "bfloat16") else torch.float32
        if c.gradient_checkpointing:
            enable_gradient_checkpointing(model)
        self.trainer = Trainer(model, TrainStepConfig(
            lr=c.learning_rate, weight_decay=c.weight_decay, betas=c.betas, grad_clip=c.max_grad_norm,
            warmup_steps=c.warmup_steps, total_steps=c.total_steps,
            gradient_accumulation_steps=c.gradient_accumulation_steps, dtype=dtype), device=device, engine=engine)
        self.model = self.trainer.model
        self.optimizer = self.trainer.optimizer

    @property
    def global_step(self) -> int:
        return self.trainer.global_step

    def train_step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        return self.trainer.train_step({"input_ids": input_ids, "labels": labels})

    def train_epoch(self, loader, log_every: int = 0, sink=print) -> float:
        total, n = None, 0
        for i, batch in enumerate(loader):
            loss = self.trainer.train_step(batch)
            total = loss if total is None else total + loss
            n += 1
            if log_every and (i + 1) % log_every == 0:
                sink(f"step {self.global_step} loss {float(loss):.4f}")
        return float(total / max(n, 1)) if total is not None else float("nan")


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
