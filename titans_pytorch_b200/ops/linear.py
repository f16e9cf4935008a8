"""Linear layers on the tcgen05 GEMM, with weight gradients accumulated in place.

``linear(x, w1, w2, ...)`` computes ``x @ [w1; w2; ...]^T`` (the weights
stacked by rows).  On CUDA with bf16 operands the three GEMMs of the layer
run on the 2-CTA tcgen05 kernel (``csrc/gemm_sm100.cu``): the forward
(``x W^T``), the input gradient (``dy W``) and the weight gradient
(``dy^T x``, split-K over the tokens with a fixed-order reduction).  Stacked
weights whose storage is adjacent (as the flat parameter buffer of the
trainer lays out q|k|v, k|v and gate|up) are read in place, with no
concatenation.

Under :func:`accumulate_weight_grads` (which the trainer turns on around its
``backward()``), the weight-gradient GEMM adds ``dy^T x`` straight into the
weights' existing ``.grad`` (accumulating epilogue) instead of returning it
to autograd, which would otherwise run a separate add kernel for every use
of the weight.  Stacked weights take the in-place path when their ``.grad``
tensors are adjacent in one buffer, as
:class:`~titans_pytorch_b200.train.optim.FlatParamSpace` lays them out.  In
every other case, and always outside the context, the gradients go back to
autograd as usual (``torch.autograd.grad`` included).

:func:`set_prefetch` installs a one-shot forward hook used by the sharded
data-parallel engine: the next ``linear`` call hands its GEMM to the hook
(which runs it on the kernel that also all-gathers the next block's
parameters) and the hook is dropped.  A hook that returns None leaves the
GEMM to the default kernel and stays installed.
"""

from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F

from . import gemm as G
from ._ext import want_kernels

_STATE = {"inplace": False, "prefetch": None, "side": None, "side_used": False}
_SIDE_STREAMS: dict[int, "torch.cuda.Stream"] = {}

# A weight gradient this small (few output tiles, a short reduction over the
# tokens) leaves most of the GPU idle on its own: MAC's per-segment GEMMs.
SIDE_MAX_TOKENS = 4096
SIDE_MAX_TILES = 36  # 256 x 256 output tiles: half of the 74 CTA pairs


def set_prefetch(fn) -> None:
    """Install (or clear, with None) the one-shot GEMM hook ``fn(x, w) -> y | None``."""
    _STATE["prefetch"] = fn


@contextlib.contextmanager
def accumulate_weight_grads(enabled: bool = True, side_stream: bool = False):
    """In-place weight gradients (see the module docstring).  ``side_stream``
    (CUDA): weight-gradient GEMMs too small to fill the GPU (at most
    ``SIDE_MAX_TOKENS`` tokens and ``SIDE_MAX_TILES`` output tiles) run on a
    second stream, so they fill the SMs that the backward's critical path
    (input gradients) leaves idle; the current stream waits for that stream
    when the context exits, before anything reads the gradients.  Callers whose
    code reads ``.grad`` inside the backward (reductions during the backward)
    must not ask for it."""
    prev = (_STATE["inplace"], _STATE["side"], _STATE["side_used"])
    _STATE["inplace"] = enabled
    side = None
    main = None
    if enabled and side_stream and torch.cuda.is_available():
        main = torch.cuda.current_stream()
        key = main.device.index
        side = _SIDE_STREAMS.get(key)
        if side is None:
            side = _SIDE_STREAMS[key] = torch.cuda.Stream(main.device)
    _STATE["side"], _STATE["side_used"] = side, False
    try:
        yield
    finally:
        if side is not None and _STATE["side_used"]:
            main.wait_stream(side)  # every weight gradient is complete from here on
        _STATE["inplace"], _STATE["side"], _STATE["side_used"] = prev


def _side_ok(dy2: torch.Tensor, target: torch.Tensor) -> bool:
    if _STATE["side"] is None or not dy2.is_cuda or dy2.shape[0] > SIDE_MAX_TOKENS:
        return False
    tiles = ((target.shape[0] + 255) // 256) * ((target.shape[1] + 255) // 256)
    return tiles <= SIDE_MAX_TILES


def inplace_grads_enabled() -> bool:
    return _STATE["inplace"]


def stacked(weights) -> torch.Tensor:
    """``cat(weights, 0)`` -- as a view of the shared storage when the weights are
    adjacent rows of one buffer (no copy), else a concatenation."""
    if len(weights) == 1:
        return weights[0]
    w0 = weights[0]
    cols = w0.shape[1] if w0.dim() == 2 else -1
    ptr, es = w0.data_ptr(), w0.element_size()
    sto = w0.untyped_storage().data_ptr()
    ok = cols > 0
    for w in weights:
        if not ok:
            break
        # same storage (not merely neighbouring allocations) and the next rows
        ok = (w.dim() == 2 and w.shape[1] == cols and w.is_contiguous() and w.dtype == w0.dtype
              and w.device == w0.device and w.data_ptr() == ptr and w.untyped_storage().data_ptr() == sto)
        ptr += w.numel() * es
    if ok:
        rows = sum(w.shape[0] for w in weights)
        base = w0.detach()
        return base.as_strided((rows, cols), (cols, 1), base.storage_offset())
    return torch.cat(weights, 0)


def grad_target(weights) -> torch.Tensor | None:
    """One [rows, cols] view covering every weight's .grad, or None."""
    g0 = weights[0].grad
    if g0 is None or not g0.is_contiguous():
        return None
    cols = weights[0].shape[1]
    ptr, es = g0.data_ptr(), g0.element_size()
    sto = g0.untyped_storage().data_ptr()
    for w in weights:
        g = w.grad
        if (g is None or not g.is_contiguous() or g.data_ptr() != ptr or w.dim() != 2 or w.shape[1] != cols
                or g.dtype != g0.dtype or g.untyped_storage().data_ptr() != sto):
            return None
        ptr += g.numel() * es
    rows = sum(w.shape[0] for w in weights)
    return g0.as_strided((rows, cols), (cols, 1), g0.storage_offset())


def mark_grads(weights) -> None:
    """The flat-buffer bookkeeping autograd's accumulation would have done."""
    for wt in weights:
        mark = getattr(wt, "_titans_grad_mark", None)
        if mark is not None:
            mark(wt)


def kernel_ok(x: torch.Tensor, w: torch.Tensor, use_kernels: bool | None = None) -> bool:
    """The tcgen05 path applies: CUDA bf16 operands the GEMM can read as they are."""
    if not (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16):
        return False
    if not want_kernels(x, use_kernels):
        return False
    K = x.shape[-1]
    return K % 8 == 0 and w.shape[0] % 8 == 0 and w.dim() == 2 and w.shape[1] == K


def _rows(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if G.operand_ok(t2) else t2.contiguous()


def _fwd(x: torch.Tensor, w: torch.Tensor, kern: bool) -> torch.Tensor:
    fn = _STATE["prefetch"]
    if fn is not None:
        y = fn(x, w)
        if y is not None:
            _STATE["prefetch"] = None
            return y
    if kern and x.numel() > 0:
        x2 = _rows(x)
        return G.mm_tn(x2, w).view(*x.shape[:-1], w.shape[0])
    return F.linear(x, w)


def weight_grads(weights, dy2: torch.Tensor, x2: torch.Tensor, kern: bool, need) -> tuple:
    """Weight gradients ``dy2^T x2`` of (stacked) ``weights``: added in place into
    adjacent ``.grad`` buffers under :func:`accumulate_weight_grads` (returns
    Nones), else returned for autograd."""
    target = grad_target(weights) if (_STATE["inplace"] and all(need)) else None
    if target is not None:
        if kern and G.operand_ok(target) and _side_ok(dy2, target):
            side = _STATE["side"]
            # The side stream reads its own copy of the output gradient: autograd may
            # later sum another contribution into the incoming gradient tensor in place
            # (when it holds the last reference), which must not race with this read.
            dy2 = dy2.clone()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                G.mm_wgrad(dy2, x2, out=target, accumulate=True)
            dy2.record_stream(side)  # the allocator must not reuse them before the side stream has read them
            x2.record_stream(side)
            _STATE["side_used"] = True
        elif kern and G.operand_ok(target):
            G.mm_wgrad(dy2, x2, out=target, accumulate=True)
        else:
            target.addmm_(dy2.t(), x2.to(dy2.dtype))
        mark_grads(weights)
        return (None,) * len(weights)
    gw = G.mm_wgrad(dy2, x2) if kern else torch.matmul(dy2.t(), x2.to(dy2.dtype))
    parts = gw.split([wt.shape[0] for wt in weights], 0) if len(weights) > 1 else (gw,)
    return tuple(g if nd else None for g, nd in zip(parts, need))


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kern, n, *weights):
        w = stacked(weights)
        ctx.save_for_backward(x, w)
        ctx.weights = weights
        ctx.kern = kern
        return _fwd(x, w, kern)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        weights, kern = ctx.weights, ctx.kern
        dy2 = _rows(dy) if kern else dy.reshape(-1, dy.shape[-1])
        dx = None
        if ctx.needs_input_grad[0]:
            dx = G.mm_nn(dy2, w).view(*dy.shape[:-1], w.shape[1]) if kern else torch.matmul(dy, w)
        need = ctx.needs_input_grad[3:]
        if not any(need):
            return (dx, None, None) + (None,) * len(weights)
        x2 = _rows(x) if kern else x.reshape(-1, x.shape[-1])
        return (dx, None, None) + weight_grads(weights, dy2, x2, kern, need)


def linear(x: torch.Tensor, *weights: torch.Tensor, use_kernels: bool | None = None) -> torch.Tensor:
    """``x @ cat(weights)^T`` (no bias).  Int8 weights (``ops.quant``) run the int8 GEMM."""
    if any(type(w).__name__ == "Int8Weight" for w in weights):
        from .quant import int8_linear

        return int8_linear(x, weights)
    kern = kernel_ok(x, weights[0], use_kernels) and all(w.dtype == torch.bfloat16 for w in weights) and all(
        w.shape[1] == x.shape[-1] and w.shape[0] % 8 == 0 for w in weights)
    if not torch.is_grad_enabled() or not any(w.requires_grad for w in weights):
        return _fwd(x, stacked(weights), kern)
    return _Linear.apply(x, kern, len(weights), *weights)


__all__ = ["linear", "accumulate_weight_grads", "set_prefetch", "stacked", "grad_target", "mark_grads",
           "kernel_ok", "weight_grads", "inplace_grads_enabled"]
