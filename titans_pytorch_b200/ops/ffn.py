"""SwiGLU feed-forward: down(silu(x Wg^T) * (x Wu^T)) [+ residual].

Reference: `src/titans/models.py:27-70` (FeedForward; its CUDA branch calls a
Triton silu*mul kernel without a backward, `triton_kernels.py:412-440`).

CUDA path (bf16): one autograd node for the whole block, four tcgen05 GEMM
launches forward+backward plus the weight gradients:

* forward: ``gu = x [Wg; Wu]^T`` with the SwiGLU in the GEMM epilogue (writes
  ``gu`` for the backward and ``h = silu(g) * u``), then ``y = h Wd^T``
  (with the residual added in the epilogue when one is given);
* backward: ``dgu`` straight from ``dy Wd`` (the SwiGLU backward is the
  epilogue of that input-gradient GEMM), ``dx = dgu [Wg; Wu]``, and the
  weight gradients ``dy^T h`` / ``dgu^T x`` (split-K, accumulated in place
  under the trainer, see ``ops.linear``).

The stacked ``[Wg; Wu]`` is a view when the two weights are adjacent in
memory (the trainer's flat parameter buffer), else a concatenation.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gemm as G
from ._ext import ext, want_kernels
from .linear import _rows, kernel_ok, linear, stacked, weight_grads


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


class _FusedFFN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, w_gate, w_up, w_down):
        x2 = _rows(x)
        w_gu = stacked((w_gate, w_up))
        gu, h = G.swiglu_fwd(x2, w_gu)
        if residual is not None:
            y = G.mm_tn(h, w_down, mode="resid", r=_rows(residual))
        else:
            y = G.mm_tn(h, w_down)
        ctx.save_for_backward(x2, gu, h, w_gu, w_down)
        ctx.weights = (w_gate, w_up, w_down)
        ctx.xshape = x.shape
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w_down.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, gu, h, w_gu, w_down = ctx.saved_tensors
        w_gate, w_up, _ = ctx.weights
        dy2 = _rows(dy)
        dgu = G.swiglu_dgrad(dy2, w_down, gu)
        need = ctx.needs_input_grad
        (gd,) = weight_grads((w_down,), dy2, h, True, (need[4],)) if need[4] else (None,)
        dx = G.mm_nn(dgu, w_gu).view(ctx.xshape) if need[0] else None
        gg, gup = weight_grads((w_gate, w_up), dgu, x2, True, (need[2], need[3])) if (need[2] or need[3]) \
            else (None, None)
        dres = dy if ctx.has_res and need[1] else None
        return dx, dres, gg, gup, gd


def swiglu_ffn(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
               dropout_p: float = 0.0, training: bool = False,
               use_kernels: bool | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``[residual +] down(silu(x Wg^T) * (x Wu^T))`` (dropout on the hidden activation in training)."""
    drop = dropout_p > 0.0 and training
    F_ = w_gate.shape[0]
    int8 = any(type(w).__name__ == "Int8Weight" for w in (w_gate, w_up, w_down))
    if (not drop and not int8 and kernel_ok(x, w_gate, use_kernels) and F_ % 32 == 0 and w_up.dtype == torch.bfloat16
            and w_down.dtype == torch.bfloat16 and w_down.shape[0] % 8 == 0 and x.numel() > 0
            and (residual is None or (residual.dtype == torch.bfloat16 and residual.shape == x.shape[:-1]
                                      + (w_down.shape[0],)))):
        return _FusedFFN.apply(x, residual, w_gate, w_up, w_down)
    if int8 and not want_kernels(x, use_kernels):
        gu = linear(x, w_gate, w_up, use_kernels=use_kernels)
        h = F.silu(gu[..., :F_]) * gu[..., F_:]
    elif want_kernels(x, use_kernels):
        gu = linear(x, w_gate, w_up, use_kernels=use_kernels)
        h = _SwiGLUFn.apply(gu.view(-1, gu.shape[-1])).view(*x.shape[:-1], F_)
    else:
        h = F.silu(F.linear(x, w_gate)) * F.linear(x, w_up)
    if drop:
        h = F.dropout(h, dropout_p, True)
    y = linear(h, w_down, use_kernels=use_kernels)
    return y if residual is None else residual + y
