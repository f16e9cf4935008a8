"""Fused softmax cross-entropy (mean over non-ignored targets).

Reference loss: ``F.cross_entropy(logits.view(-1, V), labels.view(-1))`` in
`scripts/pretrain.py:568-572`.  The CUDA path (``csrc/loss.cu``) streams each
row of logits once in the forward (online max / sum-of-exp), keeps only the
per-row log-sum-exp, and recomputes the softmax in the backward; the loss and
the valid-row count stay on the device.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, want_kernels


class _CrossEntropyFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index):
        stats, lse = ext().cross_entropy_fwd(logits, labels, ignore_index)
        ctx.save_for_backward(logits, labels, lse, stats)
        ctx.ignore_index = ignore_index
        return stats[0]

    @staticmethod
    def backward(ctx, g):
        logits, labels, lse, stats = ctx.saved_tensors
        d = ext().cross_entropy_bwd(logits, labels, lse, stats, g.reshape(1), ctx.ignore_index)
        return d, None, None


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100,
                  use_kernels: bool | None = None) -> torch.Tensor:
    """Mean cross-entropy of ``logits`` [..., V] against integer ``labels`` [...]."""
    l2 = logits.reshape(-1, logits.shape[-1])
    y = labels.reshape(-1)
    if want_kernels(l2, use_kernels):
        if l2.stride(-1) != 1:
            l2 = l2.contiguous()
        return _CrossEntropyFn.apply(l2, y, int(ignore_index))
    return F.cross_entropy(l2, y, ignore_index=ignore_index)
