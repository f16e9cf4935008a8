"""Linear layers whose weight gradient is accumulated in place.

``linear(x, w1, w2, ...)`` computes ``x @ [w1; w2; ...]^T`` (the weights
stacked by rows).  Under :func:`accumulate_weight_grads` (which the trainer
turns on around its ``backward()``), the backward adds ``dy^T x`` straight into
the weights' existing ``.grad`` with one GEMM (``addmm_``, beta = 1) instead of
returning it to autograd. Autograd would otherwise run a separate add kernel
for every use of the weight. A TitansMAC forward uses each block's weights once
per segment, so this removes one add per weight and segment. Stacked weights
take the in-place path when their ``.grad`` tensors are adjacent in one buffer,
as :class:`~titans_pytorch_b200.train.optim.FlatParamSpace` lays them out. In
every other case, and always outside the context, the gradients go back
to autograd as usual (``torch.autograd.grad`` included).

:func:`set_prefetch` installs a one-shot forward hook used by the sharded
data-parallel engine: the next ``linear`` call hands its GEMM to the hook
(which runs it on the kernel that also all-gathers the next block's
parameters) and the hook is dropped.  A hook that returns None leaves the
GEMM to cuBLAS and stays installed.
"""

from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F

_STATE = {"inplace": False, "prefetch": None}


def set_prefetch(fn) -> None:
    """Install (or clear, with None) the one-shot GEMM hook ``fn(x, w) -> y | None``."""
    _STATE["prefetch"] = fn


def _mm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    fn = _STATE["prefetch"]
    if fn is not None:
        y = fn(x, w)
        if y is not None:
            _STATE["prefetch"] = None
            return y
    return F.linear(x, w)


@contextlib.contextmanager
def accumulate_weight_grads(enabled: bool = True):
    prev = _STATE["inplace"]
    _STATE["inplace"] = enabled
    try:
        yield
    finally:
        _STATE["inplace"] = prev


def _grad_target(weights) -> torch.Tensor | None:
    """One [rows, cols] view covering every weight's .grad, or None."""
    g0 = weights[0].grad
    if g0 is None or not g0.is_contiguous():
        return None
    cols = weights[0].shape[1]
    ptr, es = g0.data_ptr(), g0.element_size()
    for w in weights:
        g = w.grad
        if (g is None or not g.is_contiguous() or g.data_ptr() != ptr or w.dim() != 2 or w.shape[1] != cols
                or g.dtype != g0.dtype):
            return None
        ptr += g.numel() * es
    rows = sum(w.shape[0] for w in weights)
    return g0.as_strided((rows, cols), (cols, 1))


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, n, *weights):
        w = weights[0] if n == 1 else torch.cat(weights, 0)
        ctx.save_for_backward(x, w)
        ctx.weights = weights
        return _mm(x, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        weights = ctx.weights
        dx = torch.matmul(dy, w) if ctx.needs_input_grad[0] else None
        need = ctx.needs_input_grad[2:]
        if not any(need):
            return (dx, None) + (None,) * len(weights)
        dy2 = dy.reshape(-1, dy.shape[-1])
        x2 = x.reshape(-1, x.shape[-1])
        target = _grad_target(weights) if (_STATE["inplace"] and all(need)) else None
        if target is not None:
            target.addmm_(dy2.t(), x2.to(dy2.dtype))
            for wt in weights:  # the flat-buffer bookkeeping autograd's accumulation would have done
                mark = getattr(wt, "_titans_grad_mark", None)
                if mark is not None:
                    mark(wt)
            return (dx, None) + (None,) * len(weights)
        gw = torch.matmul(dy2.t(), x2.to(dy2.dtype))
        parts = gw.split([wt.shape[0] for wt in weights], 0) if len(weights) > 1 else (gw,)
        return (dx, None) + tuple(g if nd else None for g, nd in zip(parts, need))


def linear(x: torch.Tensor, *weights: torch.Tensor) -> torch.Tensor:
    """``x @ cat(weights)^T`` (no bias)."""
    if not torch.is_grad_enabled() or not any(w.requires_grad for w in weights):
        w = weights[0] if len(weights) == 1 else torch.cat(weights, 0)
        return _mm(x, w)
    return _Linear.apply(x, len(weights), *weights)


__all__ = ["linear", "accumulate_weight_grads", "set_prefetch"]
