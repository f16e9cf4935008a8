"""SwiGLU feed-forward: down(silu(x Wg^T) * (x Wu^T)).

Reference: `src/titans/models.py:27-70` (FeedForward; its CUDA branch calls a
Triton silu*mul kernel without a backward, `triton_kernels.py:412-440`).

CUDA path: the gate and up projections run as ONE GEMM against the stacked
weight ``[Wg; Wu]`` and the SiLU-product is computed by the ``swiglu_fwd`` /
``swiglu_bwd`` kernels of ``csrc/elementwise.cu``.  Weight gradients go
through :func:`~titans_pytorch_b200.ops.linear.linear` (accumulated in place
under the trainer).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, want_kernels
from .linear import linear


class _SwiGLUFn(torch.autograd.Function):
    """h = silu(gu[:, :F]) * gu[:, F:] with gu the stacked gate/up output."""

    @staticmethod
    def forward(ctx, gu):
        h = ext().swiglu_fwd(gu)
        ctx.save_for_backward(gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(dh.contiguous(), gu)


def swiglu_ffn(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
               dropout_p: float = 0.0, training: bool = False,
               use_kernels: bool | None = None) -> torch.Tensor:
    if want_kernels(x, use_kernels):
        gu = linear(x, w_gate, w_up)
        h = _SwiGLUFn.apply(gu.view(-1, gu.shape[-1])).view(*x.shape[:-1], w_gate.shape[0])
    else:
        h = F.silu(F.linear(x, w_gate)) * F.linear(x, w_up)
    if dropout_p > 0.0 and training:
        h = F.dropout(h, dropout_p, True)
    return linear(h, w_down)
