"""Neural-memory math: retrieval MLP, associative-loss gradient, gated update.

Reference semantics (``semantics="ref"``), as run by the reference on CUDA:

* gradient of ``mean_{B,T,D} (MLP_W(k) - v)^2`` w.r.t. every memory weight,
  with k and v detached (`src/titans/memory.py:287-351`; CUDA branch
  `src/titans/cuda_optimizations.py:228-319`).
* one-layer memory (L_M = 1): the reference's CUDA branch has its own analytic
  form ``2/(B*T) * (silu(k) W^T - v)^T silu(k)`` (`cuda_optimizations.py:248-275`),
  but it calls ``.view`` on the keys, which are non-contiguous whenever the
  depthwise conv is on (`memory.py:263-285` transposes around the conv); the
  resulting exception sends it to the autograd fallback (`memory.py:319-346`),
  i.e. the plain mse gradient, which also switches ``requires_grad`` off on
  the memory MLP.  ``linear_silu=True`` selects the analytic form (L_M = 1,
  no conv); otherwise the plain gradient is used.
* scalar gates alpha/theta/eta: the mean over batch and channels of
  ``sigmoid(Linear(mean_T x))`` (`memory.py:427-432`).
* ``S' = eta*S - theta*G``,  ``W' = (1-alpha)*W + S'`` (`memory.py:464-498`).

The deep-memory gradient is written out as explicit back-propagation through
the MLP (no inner autograd graph).  On CUDA (bf16) every GEMM of the update
runs on the tcgen05 kernel of ``csrc/gemm_sm100.cu`` with the elementwise
work in its epilogues: the hidden layers write ``z`` and ``act(z)``, the last
layer writes the scaled error ``c (M(k) - v)``, the back-propagation GEMMs
multiply by ``act'(z)``, and each weight-gradient GEMM (split-K over the
B*T tokens, fixed-order sum) applies ``S' = eta S - theta G``,
``W' = (1 - alpha) W + S'`` to the complete gradient with the gates read on
the device -- the gradient itself is never stored, and nothing leaves the
device (no ``.item()`` host sync).  The retrieval MLP (trainable) is one
autograd node (:class:`_MemoryMLPFn`) with the activation in the forward
GEMMs' epilogues and ``act'`` in the backward GEMMs' epilogues.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import gemm as G
from ._ext import ext, want_kernels
from .linear import _rows, kernel_ok, weight_grads


def activation_fn(name: str):
    if name == "silu":
        return F.silu
    if name == "gelu":
        return F.gelu
    if name == "relu":
        return F.relu
    raise ValueError(f"Unknown activation: {name}")


class _SiLU(torch.autograd.Function):
    """silu(z) on the extension's vectorised kernels: the forward keeps z, the
    backward writes g * silu'(z) to a new tensor (one read of g and z, one write).
    Gradients the kernel cannot take (dtype other than z's, unaligned) use the
    PyTorch definition."""

    @staticmethod
    def forward(ctx, z):
        a = torch.empty_like(z)
        ext().act_inplace(z, a, "silu")
        ctx.save_for_backward(z)
        return a

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, g):
        (z,) = ctx.saved_tensors
        g = g.contiguous()
        if g.dtype != z.dtype or g.data_ptr() % 16 != 0 or g.shape != z.shape:
            return (g.float() * activation_grad("silu", z.float())).to(z.dtype)
        out = torch.empty_like(z)
        ext().act_grad_out(g, z, out, "silu")
        return out


_ACT_KERNEL = ("silu", "gelu", "relu")


class _MemoryMLPFn(torch.autograd.Function):
    """The memory MLP ``W_L act(... act(W_1 x))`` as one autograd node on the tcgen05 GEMM:
    forward GEMMs write ``z_i`` and ``act(z_i)``; the backward chains
    ``dz_{i-1} = (dz_i W_i) * act'(z_{i-1})`` (the product in the GEMM epilogue),
    ``dx = dz_1 W_1``, and the weight gradients ``dz_i^T h_{i-1}`` (in place
    under the trainer)."""

    @staticmethod
    def forward(ctx, x, act, *weights):
        x2 = _rows(x)
        hs, zs = [x2], []
        h = x2
        L = len(weights)
        for i, w in enumerate(weights):
            if i < L - 1:
                z, h = G.mm_act(h, w, act)
                zs.append(z)
                hs.append(h)
            else:
                h = G.mm_tn(h, w)
        ctx.save_for_backward(*hs, *zs)
        ctx.weights = weights
        ctx.act = act
        ctx.xshape = x.shape
        return h.view(*x.shape[:-1], weights[-1].shape[0])

    @staticmethod
    def backward(ctx, dy):
        weights, act = ctx.weights, ctx.act
        L = len(weights)
        saved = ctx.saved_tensors
        hs, zs = saved[:L], saved[L:]
        need = ctx.needs_input_grad[2:]
        d = _rows(dy)
        grads = [None] * L
        dx = None
        for i in range(L - 1, -1, -1):
            nd = None
            if i > 0:
                nd = G.mm_act_grad(d, weights[i], zs[i - 1], act)
            elif ctx.needs_input_grad[0]:
                dx = G.mm_nn(d, weights[0]).view(ctx.xshape)
            if need[i]:
                (grads[i],) = weight_grads((weights[i],), d, hs[i], True, (True,))
            d = nd
        return (dx, None) + tuple(grads)


def mlp_kernel_ok(x: torch.Tensor, weights, act: str, use_kernels: bool | None = None) -> bool:
    """The fused tcgen05 memory-MLP path applies (bf16 CUDA, GEMM-compatible sizes)."""
    if act not in _ACT_KERNEL or x.numel() == 0:
        return False
    if not kernel_ok(x, weights[0], use_kernels):
        return False
    return all(w.dtype == torch.bfloat16 and w.dim() == 2 and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0
               for w in weights)


def memory_mlp(x: torch.Tensor, weights, act: str) -> torch.Tensor:
    """``MLP_W(x)`` on the fused tcgen05 path (callers check :func:`mlp_kernel_ok`)."""
    if torch.is_grad_enabled() and (x.requires_grad or any(w.requires_grad for w in weights)):
        return _MemoryMLPFn.apply(x, act, *weights)
    x2 = _rows(x)
    h = x2
    for i, w in enumerate(weights):
        h = G.mm_act(h, w, act, keep_z=False)[1] if i < len(weights) - 1 else G.mm_tn(h, w)
    return h.view(*x.shape[:-1], weights[-1].shape[0])


def activation(z: torch.Tensor, name: str, use_kernels: bool | None = None) -> torch.Tensor:
    """``act(z)``; SiLU on CUDA (bf16 / fp32, contiguous, 16-byte aligned) runs the
    extension's kernels, everything else ``activation_fn(name)``."""
    if (name == "silu" and want_kernels(z, use_kernels) and z.dtype in (torch.bfloat16, torch.float32)
            and z.is_contiguous() and z.numel() % (16 // z.element_size()) == 0 and z.data_ptr() % 16 == 0):
        return _SiLU.apply(z)
    return activation_fn(name)(z)


def activation_grad(name: str, z: torch.Tensor) -> torch.Tensor:
    """d act(z) / dz, elementwise."""
    if name == "silu":
        s = torch.sigmoid(z)
        return s * (1 + z * (1 - s))
    if name == "gelu":  # exact (erf) GELU, nn.GELU's default
        return 0.5 * (1 + torch.erf(z / math.sqrt(2.0))) + z * torch.exp(-0.5 * z * z) / math.sqrt(2 * math.pi)
    if name == "relu":
        return (z > 0).to(z.dtype)
    raise ValueError(f"Unknown activation: {name}")


def mlp_forward_reference(x: torch.Tensor, weights: list[torch.Tensor], act: str) -> torch.Tensor:
    h = x
    f = activation_fn(act)
    for i, w in enumerate(weights):
        h = F.linear(h, w)
        if i < len(weights) - 1:
            h = f(h)
    return h


def memory_grads_reference(k: torch.Tensor, v: torch.Tensor, weights: list[torch.Tensor],
                           act: str, linear_silu: bool = False) -> list[torch.Tensor]:
    """Gradient of the associative-memory loss for every memory weight (ref semantics)."""
    B, T, D = k.shape
    f = activation_fn(act)
    k2 = k.reshape(-1, D)
    v2 = v.reshape(-1, v.shape[-1])
    if len(weights) == 1 and linear_silu:
        h = f(k2)
        diff = F.linear(h, weights[0]) - v2
        return [(diff.t() @ h) * (2.0 / (B * T))]
    hs = [k2]
    zs = []
    h = k2
    for i, w in enumerate(weights):
        z = F.linear(h, w)
        if i < len(weights) - 1:
            zs.append(z)
            h = f(z)
            hs.append(h)
        else:
            h = z
    delta = (h - v2) * (2.0 / h.numel())
    grads = [None] * len(weights)
    for i in range(len(weights) - 1, -1, -1):
        grads[i] = delta.t() @ hs[i]
        if i > 0:
            delta = (delta @ weights[i]) * activation_grad(act, zs[i - 1])
    return grads


def memory_gates_reference(x_mean: torch.Tensor, gate_ws, gate_bs, lr: float, mom: float):
    """(alpha, theta, eta) as 0-dim tensors from ``x_mean`` [B, 1, D]."""
    a = torch.sigmoid(F.linear(x_mean, gate_ws[0], gate_bs[0])).mean()
    t = torch.sigmoid(F.linear(x_mean, gate_ws[1], gate_bs[1])).mean() * lr
    e = torch.sigmoid(F.linear(x_mean, gate_ws[2], gate_bs[2])).mean() * mom
    return a, t, e


def memory_update_reference(weights, momentum, grads, alpha, eta, theta):
    new_m = [eta * m - theta * g for m, g in zip(momentum, grads, strict=True)]
    new_w = [(1 - alpha) * w + s for w, s in zip(weights, new_m, strict=True)]
    return new_w, new_m


@torch.no_grad()
def memory_step(k: torch.Tensor, v: torch.Tensor, x_for_gates: torch.Tensor,
                weights: list[torch.Tensor], momentum: list[torch.Tensor],
                gate_ws, gate_bs, lr: float, mom: float, act: str,
                linear_silu: bool = False, use_kernels: bool | None = None):
    """One reference-semantics memory update; returns (new_weights, new_momentum).

    ``k`` and ``v`` are the (already conv/SiLU/L2-processed) keys and values,
    ``x_for_gates`` the memory input whose sequence mean drives the gates.
    Nothing here is differentiated (the reference detaches k, v and the new
    state, `memory.py:330-331, 461`).
    """
    if want_kernels(k, use_kernels):
        return _memory_step_cuda(k, v, x_for_gates, weights, momentum, gate_ws, gate_bs,
                                 lr, mom, act, linear_silu)
    x_mean = x_for_gates.float().mean(dim=1, keepdim=True).to(x_for_gates.dtype)
    alpha, theta, eta = memory_gates_reference(x_mean, gate_ws, gate_bs, lr, mom)
    grads = memory_grads_reference(k, v, weights, act, linear_silu)
    return memory_update_reference(weights, momentum, grads, alpha, eta, theta)


def _fused_update_ok(k2, v2, weights, momentum, act) -> bool:
    if k2.dtype != torch.bfloat16 or v2.dtype != torch.bfloat16 or act not in _ACT_KERNEL:
        return False
    if not (G.operand_ok(k2) and G.operand_ok(v2)):
        return False
    for w, m in zip(weights, momentum, strict=True):
        # the weights are GEMM operands (bf16); the momentum shares their dtype
        if (w.dtype != torch.bfloat16 or m.dtype != w.dtype or w.dim() != 2 or not w.is_contiguous()
                or not m.is_contiguous() or w.shape[0] % 8 or w.shape[1] % 8):
            return False
    return True


def _memory_step_fused(k2, v2, weights, momentum, gates, act, linear_silu, B, T):
    """The update on the tcgen05 GEMM: forward with act epilogues, error
    epilogue, back-propagation with act' epilogues, and the gated update in
    the epilogue of each (split-K) weight-gradient GEMM."""
    L = len(weights)
    if L == 1 and linear_silu:
        h = torch.empty_like(k2)
        ext().act_inplace(k2, h, act)
        delta = G.mm_err(h, weights[0], v2, 2.0 / (B * T))
        w2, m2 = G.mm_mem_update(delta, h, weights[0], momentum[0], gates)
        return [w2], [m2]
    hs, zs = [k2], []
    h = k2
    for i, w in enumerate(weights[:-1]):
        z, h = G.mm_act(h, w, act)
        zs.append(z)
        hs.append(h)
    delta = G.mm_err(h, weights[-1], v2, 2.0 / (k2.shape[0] * weights[-1].shape[0]))
    new_w, new_m = [None] * L, [None] * L
    for i in range(L - 1, -1, -1):
        nd = G.mm_act_grad(delta, weights[i], zs[i - 1], act) if i > 0 else None  # old W_i
        new_w[i], new_m[i] = G.mm_mem_update(delta, hs[i], weights[i], momentum[i], gates)
        delta = nd
    return new_w, new_m


def _memory_grads_cuda(k2, v2, weights, act, linear_silu, B, T):
    """fp32 associative-loss gradients with PyTorch GEMMs and the extension's epilogue kernels."""
    E = ext()
    L = len(weights)
    if L == 1 and linear_silu:
        h = torch.empty_like(k2)
        E.act_inplace(k2, h, act)
        pred = torch.mm(h, weights[0].t())
        E.scaled_err(pred, v2, 2.0 / (B * T))
        return [torch.mm(pred.t(), h, out_dtype=torch.float32)]
    hs, zs = [k2], []
    h = k2
    for i, w in enumerate(weights):
        z = torch.mm(h, w.t())
        if i < L - 1:
            a = torch.empty_like(z)
            E.act_inplace(z, a, act)
            zs.append(z)
            hs.append(a)
            h = a
        else:
            h = z
    E.scaled_err(h, v2, 2.0 / h.numel())
    delta = h
    grads = [None] * L
    for i in range(L - 1, -1, -1):
        grads[i] = torch.mm(delta.t(), hs[i], out_dtype=torch.float32)
        if i > 0:
            nd = torch.mm(delta, weights[i])
            E.act_grad_mul(nd, zs[i - 1], act)
            delta = nd
    return grads


def _memory_grads_tc(k2, v2, weights, act, linear_silu, B, T):
    """fp32 associative-loss gradients on the tcgen05 GEMM: the fused update's
    forward (act epilogues), error and act' back-propagation, with the weight
    gradients stored in fp32 instead of applied (the caller reduces them first)."""
    L = len(weights)
    if L == 1 and linear_silu:
        h = torch.empty_like(k2)
        ext().act_inplace(k2, h, act)
        return [G.mm_wgrad(G.mm_err(h, weights[0], v2, 2.0 / (B * T)), h, fp32=True)]
    hs, zs = [k2], []
    h = k2
    for w in weights[:-1]:
        z, h = G.mm_act(h, w, act)
        zs.append(z)
        hs.append(h)
    delta = G.mm_err(h, weights[-1], v2, 2.0 / (k2.shape[0] * weights[-1].shape[0]))
    grads = [None] * L
    for i in range(L - 1, -1, -1):
        grads[i] = G.mm_wgrad(delta, hs[i], fp32=True)
        if i > 0:
            delta = G.mm_act_grad(delta, weights[i], zs[i - 1], act)
    return grads


def _flat_kv(k, v):
    D = k.shape[-1]
    k2 = k.reshape(-1, D)
    v2 = v.reshape(-1, v.shape[-1])
    return (k2 if k2.is_contiguous() else k2.contiguous()), (v2 if v2.is_contiguous() else v2.contiguous())


def _apply_update(weights, momentum, grads, gates):
    E = ext()
    new_w, new_m = [], []
    for w, m, g in zip(weights, momentum, grads, strict=True):
        w2, m2 = E.mem_update(w, m, g, gates)
        new_w.append(w2)
        new_m.append(m2)
    return new_w, new_m


def _memory_step_cuda(k, v, x_for_gates, weights, momentum, gate_ws, gate_bs, lr, mom, act,
                      linear_silu):
    """Device-resident update: gates kernel, then the fused tcgen05 path (bf16)
    or PyTorch GEMMs with the extension's epilogue kernels."""
    E = ext()
    gates = E.memory_gates(x_for_gates, list(gate_ws), list(gate_bs), float(lr), float(mom))
    B, T, _ = k.shape
    k2, v2 = _flat_kv(k, v)
    if _fused_update_ok(k2, v2, weights, momentum, act) and want_kernels(k2):
        return _memory_step_fused(k2, v2, list(weights), list(momentum), gates, act, linear_silu, B, T)
    return _apply_update(weights, momentum, _memory_grads_cuda(k2, v2, weights, act, linear_silu, B, T), gates)


@torch.no_grad()
def memory_step_sharded(k, v, x_for_gates, weights, momentum, gate_ws, gate_bs, lr: float, mom: float,
                        act: str, linear_silu: bool, use_kernels, shard):
    """:func:`memory_step` of a sequence split over the ranks of ``shard``
    (a :class:`titans_pytorch_b200.parallel.context.ContextShard`).

    Each rank holds ``T`` of the sequence's tokens.  The gates read the mean of
    the memory input over the whole sequence and the gradient is the mean of
    per-token terms over the whole sequence; with equal shards both are the
    average over ranks of the shard's own value, so one all-reduce of both (in
    one fp32 buffer) gives every rank the state the unsharded update computes.
    """
    x_mean = x_for_gates.float().mean(dim=1, keepdim=True)
    B, T, _ = k.shape
    cuda = want_kernels(k, use_kernels)
    if cuda:
        k2, v2 = _flat_kv(k, v)
        tc = _fused_update_ok(k2, v2, weights, momentum, act)
        grads = (_memory_grads_tc if tc else _memory_grads_cuda)(k2, v2, weights, act, linear_silu, B, T)
    else:
        grads = [g.float() for g in memory_grads_reference(k, v, weights, act, linear_silu)]
    parts = [x_mean] + grads
    flat = torch.cat([t.reshape(-1) for t in parts])
    shard.all_reduce_mean_(flat)
    x_mean, *grads = [t.view_as(g) for t, g in zip(flat.split([t.numel() for t in parts]), parts, strict=True)]
    x_mean = x_mean.to(x_for_gates.dtype)
    if cuda:
        gates = ext().memory_gates(x_mean, list(gate_ws), list(gate_bs), float(lr), float(mom))
        return _apply_update(weights, momentum, grads, gates)
    alpha, theta, eta = memory_gates_reference(x_mean, gate_ws, gate_bs, lr, mom)
    grads = [g.to(w.dtype) for g, w in zip(grads, weights, strict=True)]
    return memory_update_reference(weights, momentum, grads, alpha, eta, theta)
