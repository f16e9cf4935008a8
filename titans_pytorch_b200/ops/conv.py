"""Causal depthwise conv1d fused with SiLU and an optional row L2-normalisation.

Reference: the memory's key/value/query path `src/titans/memory.py:263-285`
(``Conv1d(groups=D, padding=K-1)[..., :T]``), then ``F.silu`` (`:414-416`) and
``F.normalize(p=2, dim=-1)`` for queries and keys (`:419-420`).  On CUDA one
kernel (``csrc/conv.cu``) computes conv + bias + SiLU + L2 norm per row; the
backward recomputes the forward in registers instead of saving activations.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, want_kernels

L2_EPS = 1e-12  # F.normalize default


def causal_dwconv_reference(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    """y[t, d] = b[d] + sum_j w[d, 0, j] * x[t - K + 1 + j, d] (zero before t=0)."""
    k = w.shape[-1]
    xt = F.pad(x.transpose(1, 2), (k - 1, 0))
    return F.conv1d(xt, w, b, groups=x.shape[-1]).transpose(1, 2)


def conv_silu_norm_reference(x, w, b, normalize: bool):
    y = causal_dwconv_reference(x, w, b) if w is not None else x
    y = F.silu(y)
    if normalize:
        y = F.normalize(y, p=2, dim=-1, eps=L2_EPS)
    return y


class _ConvSiluNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, normalize):
        y = ext().conv_silu_norm_fwd(x, w, b, bool(normalize))
        ctx.save_for_backward(x, w, b)
        ctx.normalize = bool(normalize)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, b = ctx.saved_tensors
        dx, dw, db = ext().conv_silu_norm_bwd(dy.contiguous(), x, w, b, ctx.normalize,
                                              ctx.needs_input_grad[1] and w is not None)
        dw = dw.view_as(w).to(w.dtype) if (w is not None and dw.numel()) else None
        db = db.to(b.dtype) if (b is not None and db.numel()) else None
        return dx, dw, db, None


def conv_silu_norm(x: torch.Tensor, w: torch.Tensor | None, b: torch.Tensor | None,
                   normalize: bool, use_kernels: bool | None = None) -> torch.Tensor:
    """silu(causal_dwconv(x)) [then L2-normalised over the last dim].

    ``x`` is ``[B, T, D]`` (the last dim must be contiguous; the row stride may
    be larger than D, e.g. a slice of a fused projection output).  ``w`` is
    ``[D, 1, K]`` or ``None`` (no convolution).
    """
    if want_kernels(x, use_kernels):
        return _ConvSiluNormFn.apply(x, w, b, normalize)
    return conv_silu_norm_reference(x, w, b, normalize)
