"""Weight-only int8 inference: int8 weights in memory, dequantised inside the GEMM.

The reference's int8 path (`src/titans/optimized_inference.py:481-536`,
`scripts/inference.py:168-219`) applies torch's dynamic quantisation to
``nn.Linear`` modules (CPU only).  Here :func:`quantize_model_int8` replaces
the bias-free ``nn.Linear`` weights of a model by :class:`Int8Weight`: int8
rows with one fp32 scale per output row (symmetric, round to nearest), half
the bf16 bytes.  ``ops.linear`` routes such weights to
``csrc/quant.cu``: up to 16 activation rows (token-by-token decoding) run the
int8 GEMM that dequantises the weight bytes in registers inside its K loop;
larger inputs dequantise into a transient bf16 weight and run the tcgen05
GEMM.  Any other operation on an :class:`Int8Weight` sees the dequantised
tensor (``__torch_dispatch__``), so code that reads a weight directly stays
correct.

Left in bf16: the memory MLP (its weights are overwritten with the memory
state at every forward), layers with a bias (the memory gates), and the
embedding table (a tied output head gets its own int8 copy).
"""

from __future__ import annotations

import torch
import torch.nn as nn
from torch.utils import _pytree as pytree

from ._ext import ext

_STACKED: dict[tuple[int, ...], "Int8Weight"] = {}


def quantize_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(int8 rows, fp32 row scales) of a [N, K] weight."""
    if w.is_cuda and w.dtype == torch.bfloat16 and w.is_contiguous():
        q, s = ext().quantize_int8_rows(w)
        return q, s
    wf = w.detach().float()
    s = wf.abs().amax(dim=1).clamp_min(0.0)
    s = torch.where(s > 0, s / 127.0, torch.ones_like(s))
    q = torch.round(wf / s[:, None]).clamp_(-127, 127).to(torch.int8)
    return q, s


class Int8Weight(torch.Tensor):
    """A [N, K] weight that presents as ``dtype`` but is stored as int8 rows + scales."""

    @staticmethod
    def __new__(cls, q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.bfloat16):
        t = torch.Tensor._make_wrapper_subclass(cls, q.shape, dtype=dtype, device=q.device, requires_grad=False)
        t.q = q
        t.scale = scale
        return t

    def __init__(self, q, scale, dtype=torch.bfloat16):  # noqa: D107 (state set in __new__)
        super().__init__()

    def __repr__(self) -> str:
        return f"Int8Weight(shape={tuple(self.shape)}, dtype={self.dtype}, device={self.device})"

    def nbytes_stored(self) -> int:
        return self.q.numel() * self.q.element_size() + self.scale.numel() * self.scale.element_size()

    def dequantize(self) -> torch.Tensor:
        if self.q.is_cuda and self.dtype == torch.bfloat16 and self.q.shape[1] % 16 == 0:
            return ext().dequantize_int8_rows(self.q, self.scale)
        return (self.q.float() * self.scale[:, None]).to(self.dtype)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        if func is torch.ops.aten.detach.default:
            return args[0]

        def unwrap(t):
            return t.dequantize() if isinstance(t, Int8Weight) else t

        return func(*pytree.tree_map(unwrap, args), **pytree.tree_map(unwrap, kwargs or {}))


def _stacked(weights) -> Int8Weight:
    if len(weights) == 1:
        return weights[0]
    key = tuple(id(w) for w in weights)
    st = _STACKED.get(key)
    if st is None:
        st = Int8Weight(torch.cat([w.q for w in weights], 0), torch.cat([w.scale for w in weights], 0),
                        weights[0].dtype)
        _STACKED[key] = st
    return st


def int8_linear(x: torch.Tensor, weights) -> torch.Tensor:
    """``x @ cat(weights)^T`` for :class:`Int8Weight` weights (no autograd)."""
    ws = [w if isinstance(w, Int8Weight) else Int8Weight(*quantize_rows(w.detach()), w.dtype) for w in weights]
    w = _stacked(ws)
    N, K = w.shape
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if (x2.is_cuda and x2.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and 0 < M <= 16 and K % 16 == 0
            and x2.stride(-1) == 1 and x2.stride(0) % 8 == 0 and x2.data_ptr() % 16 == 0):
        y = ext().int8_gemm_small(x2, w.q, w.scale)
    else:
        from .linear import linear

        y = linear(x2.contiguous(), w.dequantize())  # transient bf16 weight, tensor-core GEMM
    return y.view(*x.shape[:-1], N)


def _is_int8(w) -> bool:
    return isinstance(w, Int8Weight)


@torch.no_grad()
def quantize_model_int8(model: nn.Module) -> nn.Module:
    """Replace the model's bias-free ``nn.Linear`` weights by :class:`Int8Weight`
    (except the memory MLP); frees their bf16 storage.  For inference."""
    from ..models.memory import MemoryMLP

    skip = {id(p) for m in model.modules() if isinstance(m, MemoryMLP) for p in m.parameters()}
    done: dict[int, Int8Weight] = {}
    for mod in model.modules():
        if not isinstance(mod, nn.Linear) or mod.bias is not None:
            continue
        w = mod.weight
        if isinstance(w, Int8Weight) or id(w) in skip:
            continue
        qw = done.get(id(w))
        if qw is None:
            q, s = quantize_rows(w.detach().contiguous())
            qw = Int8Weight(q, s, w.dtype)
            done[id(w)] = qw
        del mod._parameters["weight"]
        mod.weight = qw
    _STACKED.clear()
    return model


def int8_weight_bytes(model: nn.Module) -> int:
    """Bytes held by the model's int8 weights (rows + scales)."""
    seen, total = set(), 0
    for mod in model.modules():
        w = getattr(mod, "weight", None)
        if isinstance(w, Int8Weight) and id(w) not in seen:
            seen.add(id(w))
            total += w.nbytes_stored()
    return total


__all__ = ["Int8Weight", "quantize_model_int8", "quantize_rows", "int8_linear", "int8_weight_bytes"]
