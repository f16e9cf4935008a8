"""RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w.

Reference: `src/titans/models.py:73-136` (RMSNorm; its CUDA branch calls a
Triton kernel with no backward, `triton_kernels.py:375-410`).  Here the CUDA
path is a fused forward/backward pair in ``csrc/norm.cu``: one warp-per-row
pass that reads x once, keeps the row in registers and writes y plus the
fp32 reciprocal RMS used by the backward.
"""

from __future__ import annotations

import torch

from ._ext import ext, want_kernels


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    rms = torch.sqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)
    return x / rms * weight


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        y, rstd = ext().rms_norm_fwd(x2, weight, float(eps))
        ctx.save_for_backward(x2, weight, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.stride(-1) != 1:
            dy2 = dy2.contiguous()
        dx, dw = ext().rms_norm_bwd(dy2, x2, weight, rstd, ctx.needs_input_grad[1])
        return dx.view(ctx.shape), (dw.to(weight.dtype) if dw is not None and dw.numel() else None), None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
             use_kernels: bool | None = None) -> torch.Tensor:
    """RMS-normalise the last dimension of ``x`` and scale by ``weight``."""
    if want_kernels(x, use_kernels):
        return _RMSNormFn.apply(x, weight, eps)
    return rms_norm_reference(x, weight, eps)


def fused_add_rms_norm_reference(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    hidden = x + residual
    return hidden, rms_norm_reference(hidden, weight, eps)


class _AddRMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, residual, weight, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        r2 = residual.reshape(-1, shape[-1]).to(x.dtype).contiguous()
        h, y, rstd = ext().rms_norm_add_fwd(x2, r2, weight, float(eps))
        ctx.save_for_backward(h, weight, rstd)
        ctx.shape = shape
        return h.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, weight, rstd = ctx.saved_tensors
        D = ctx.shape[-1]
        dy2 = torch.zeros_like(h) if dy is None else dy.reshape(-1, D).contiguous()
        dh2 = None if dh is None else dh.reshape(-1, D).to(h.dtype).contiguous()
        dx, dw = ext().rms_norm_bwd(dy2, h, weight, rstd, ctx.needs_input_grad[2], dh2)
        dw = dw.to(weight.dtype) if dw is not None and dw.numel() else None
        dx = dx.view(ctx.shape)
        return dx, dx, dw, None


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                       use_kernels: bool | None = None):
    """``hidden = x + residual`` and ``rms_norm(hidden) * weight`` in one pass.

    Returns ``(hidden, normalized)`` (the reference's
    `cuda_optimizations.py:106-122` contract).  On CUDA one kernel reads both
    inputs once and writes both outputs; the backward is one kernel that also
    adds the gradient arriving at ``hidden``.
    """
    if want_kernels(x, use_kernels):
        return _AddRMSNormFn.apply(x, residual, weight, eps)
    return fused_add_rms_norm_reference(x, residual, weight, eps)
