"""RMSNorm and the SwiGLU feed-forward block.

Parameter names match the reference (`src/titans/models.py:27-136`):
``norm.weight``; ``ffn.gate_proj.weight``, ``ffn.up_proj.weight``,
``ffn.down_proj.weight``.  Unlike the reference's CUDA path, both layers are
differentiable on the GPU (the reference's raw Triton calls drop the
gradient, `models.py:61-63, 105-111`).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..config import TitansConfig
from ..ops.ffn import swiglu_ffn
from ..ops.norm import fused_add_rms_norm, rms_norm


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, use_kernels: bool | None = None) -> None:
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.use_kernels = use_kernels
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps, self.use_kernels)

    def forward_with_residual(self, x: torch.Tensor, residual: torch.Tensor):
        """(h, norm(h)) with h = x + residual (one fused kernel on CUDA)."""
        return fused_add_rms_norm(x, residual, self.weight, self.eps, self.use_kernels)


class FeedForward(nn.Module):
    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.dim = config.dim
        self.hidden_dim = config.ffn_dim
        self.use_kernels = config.use_kernels
        self.gate_proj = nn.Linear(config.dim, config.ffn_dim, bias=False)
        self.up_proj = nn.Linear(config.dim, config.ffn_dim, bias=False)
        self.down_proj = nn.Linear(config.ffn_dim, config.dim, bias=False)
        self.dropout = nn.Dropout(config.dropout)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``ffn(x)``, or ``residual + ffn(x)`` with the add fused into the down projection
        (the caller's dropout on the FFN output must be inactive to pass ``residual``)."""
        return swiglu_ffn(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight,
                          self.dropout.p, self.training, self.use_kernels, residual=residual)
