"""Paper-semantics neural memory: independent memories with per-token gates and
the chunked parallel update of the Titans paper (Behrouz, Zhong, Mirrokni 2024,
section 3.2, "Parallelize the long-term memory training").

There are N independent memories (one per sample and head).  A memory is an
MLP M_W: R^d -> R^d with weights W = (W_1, ..., W_L) (``W_l`` is
``[out, in]``); the associative loss of token t is
``l_t(W) = mean_j (M_W(k_t)_j - v_{t,j})^2``.  The sequence is cut into chunks
of C tokens.  Inside a chunk every per-token gradient is taken at the weights
W_0 the chunk starts from (the paper's chunked approximation), and the
momentum / decay recurrence with per-token gates

    S_t = eta_t S_{t-1} - theta_t u_t,   W_t = (1 - alpha_t) W_{t-1} + S_t,
    u_t = grad_W l_t(W_0),  t = 1..C

is folded into scalars:

    W_C = A W_0 + b S_0 - sum_t c_t u_t,     S_C = p S_0 - sum_t d_t u_t

    a_t = prod_{s>t} (1 - alpha_s),  A = prod_s (1 - alpha_s),  E_t = prod_{s<=t} eta_s,
    p = E_C,  b = sum_t a_t E_t,  d_t = theta_t prod_{s>t} eta_s,
    c_t = theta_t F_t,  F_t = sum_{r>=t} a_r prod_{t<s<=r} eta_s  (F_t = a_t + eta_{t+1} F_{t+1}).

For layer l, u_t is the outer product delta_l[t] h_l[t]^T (delta_l: the
loss gradient at the layer's output, h_l: its input), so
``sum_t c_t u_t = delta_l^T diag(c) h_l``: two weighted weight-gradient GEMMs
per layer and chunk.  The queries of a chunk read the memory W_0 (before the
chunk's update).

This module is the plain-PyTorch statement of that math (vectorised over the
N memories, looped over chunks).  It is the numerical oracle of the fused
sm_100a kernel and the CPU path of ``semantics="paper"``.
"""

from __future__ import annotations

import torch

from .memory import activation_fn, activation_grad


def chunk_coefficients(theta: torch.Tensor, eta: torch.Tensor, alpha: torch.Tensor):
    """Fold one chunk's recurrence into (A, b, c, p, d).

    ``theta``, ``eta``, ``alpha``: ``[..., C]`` (fp32).  Returns A, b, p of
    shape ``[...]`` and c, d of shape ``[..., C]``.  The triangular sums use
    differences of cumulative log-products (every exponent is <= 0), so nothing
    overflows for long chunks.
    """
    C = theta.shape[-1]
    tiny = torch.finfo(torch.float32).tiny
    la = torch.log((1.0 - alpha).clamp_min(tiny))
    le = torch.log(eta.clamp_min(tiny))
    cla = torch.cumsum(la, -1)                       # sum_{s<=t} log(1 - alpha_s)
    cle = torch.cumsum(le, -1)                       # log E_t
    log_a = cla[..., -1:] - cla                      # log prod_{s>t} (1 - alpha_s)
    a = torch.exp(log_a)
    A = torch.exp(cla[..., -1])
    p = torch.exp(cle[..., -1])
    b = (a * torch.exp(cle)).sum(-1)
    d = theta * torch.exp(cle[..., -1:] - cle)       # theta_t prod_{s>t} eta_s
    # F_t = sum_{r>=t} a_r exp(cle_r - cle_t)
    diff = cle.unsqueeze(-2) - cle.unsqueeze(-1)     # [..., t, r] = cle_r - cle_t
    upper = torch.ones(C, C, dtype=torch.bool, device=theta.device).triu()
    M = torch.where(upper, torch.exp(diff.clamp_max(0.0)), torch.zeros((), device=theta.device))
    F = (M * a.unsqueeze(-2)).sum(-1)
    return A, b, theta * F, p, d


def _mlp_forward(x: torch.Tensor, weights: list[torch.Tensor], act: str):
    """x: [N, C, in]; weights: [N, out, in].  Returns layer inputs and pre-activations."""
    f = activation_fn(act)
    hs, zs = [x], []
    for i, w in enumerate(weights):
        z = torch.bmm(hs[-1], w.transpose(1, 2))
        zs.append(z)
        hs.append(f(z) if i < len(weights) - 1 else z)
    return hs, zs


def _mlp_backward(delta: torch.Tensor, weights: list[torch.Tensor], zs: list[torch.Tensor], act: str):
    """Loss gradients at every layer's output, last layer first reversed back to input order."""
    deltas = [delta]
    for i in range(len(weights) - 1, 0, -1):
        dh = torch.bmm(deltas[0], weights[i])
        deltas.insert(0, dh * activation_grad(act, zs[i - 1]))
    return deltas


def memory_scan_reference(weights: list[torch.Tensor], momentum: list[torch.Tensor], k: torch.Tensor,
                          v: torch.Tensor, q: torch.Tensor | None, theta: torch.Tensor, eta: torch.Tensor,
                          alpha: torch.Tensor, chunk: int, act: str = "silu", dy: torch.Tensor | None = None):
    """Chunked memory scan over the whole sequence.

    weights / momentum: lists of ``[N, out, in]``; k, v, q: ``[N, T, d]``;
    theta, eta, alpha: ``[N, T]``.  ``dy`` (``[N, T, d]``, optional) is the
    gradient of the retrieval output; with it the function also returns the
    gradient of q (the memory weights are constants for the outer loss).
    Returns ``(y, new_weights, new_momentum, dq)`` with y = retrieval of q.
    """
    N, T, d = k.shape
    f32 = torch.float64 if k.dtype == torch.float64 else torch.float32
    W = [w.to(f32).clone() for w in weights]
    S = [m.to(f32).clone() for m in momentum]
    k, v = k.to(f32), v.to(f32)
    q = None if q is None else q.to(f32)
    dy = None if dy is None else dy.to(f32)
    ys, dqs = [], []
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        kc, vc = k[:, c0:c1], v[:, c0:c1]
        if q is not None:
            hq, zq = _mlp_forward(q[:, c0:c1], W, act)
            ys.append(hq[-1])
            if dy is not None:
                dq = _mlp_backward(dy[:, c0:c1], W, zq, act)[0]
                dqs.append(torch.bmm(dq, W[0]))
        hs, zs = _mlp_forward(kc, W, act)
        delta = 2.0 * (hs[-1] - vc) / d
        deltas = _mlp_backward(delta, W, zs, act)
        A, b, c, p, dd = chunk_coefficients(theta[:, c0:c1].to(f32), eta[:, c0:c1].to(f32),
                                            alpha[:, c0:c1].to(f32))
        for i in range(len(W)):
            gc = torch.bmm((deltas[i] * c.unsqueeze(-1)).transpose(1, 2), hs[i])
            gd = torch.bmm((deltas[i] * dd.unsqueeze(-1)).transpose(1, 2), hs[i])
            Wn = A[:, None, None] * W[i] + b[:, None, None] * S[i] - gc
            S[i] = p[:, None, None] * S[i] - gd
            W[i] = Wn
    y = torch.cat(ys, 1) if ys else None
    dq = torch.cat(dqs, 1) if dqs else None
    return y, W, S, dq


def memory_recurrence_tokenwise(weights, momentum, k, v, theta, eta, alpha, chunk: int, act: str = "silu"):
    """The same update written token by token (gradients still at each chunk's
    start weights): the unfolded recurrence that ``chunk_coefficients`` folds.
    Test oracle only."""
    N, T, d = k.shape
    W = [w.double().clone() for w in weights]
    S = [m.double().clone() for m in momentum]
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        W0 = [w.clone() for w in W]
        hs, zs = _mlp_forward(k[:, c0:c1].double(), W0, act)
        delta = 2.0 * (hs[-1] - v[:, c0:c1].double()) / d
        deltas = _mlp_backward(delta, W0, zs, act)
        for t in range(c1 - c0):
            for i in range(len(W)):
                u = deltas[i][:, t, :, None] * hs[i][:, t, None, :]
                S[i] = eta[:, c0 + t, None, None].double() * S[i] - theta[:, c0 + t, None, None].double() * u
                W[i] = (1 - alpha[:, c0 + t, None, None].double()) * W[i] + S[i]
    return W, S


def scan_kernel_supported(weights: list[torch.Tensor], k: torch.Tensor, chunk: int, act: str) -> bool:
    """Shapes the fused sm_100a scan handles: 2-layer memories of width 64 and
    hidden 256, chunks of 64, SiLU."""
    return (len(weights) == 2 and tuple(weights[0].shape[1:]) == (256, 64) and
            tuple(weights[1].shape[1:]) == (64, 256) and k.shape[-1] == 64 and chunk == 64 and act == "silu")


def memory_scan(weights: list[torch.Tensor], momentum: list[torch.Tensor], k: torch.Tensor, v: torch.Tensor,
                q: torch.Tensor, theta: torch.Tensor, eta: torch.Tensor, alpha: torch.Tensor, chunk: int,
                act: str = "silu", use_kernels: bool | None = None):
    """Retrieval outputs and final state of the chunked scan (no autograd).

    On CUDA with a supported shape this is one launch of the fused scan
    kernel (bf16 tensor-core operands, fp32 state); otherwise the PyTorch
    statement above.  Returns ``(y, new_weights, new_momentum)``.
    """
    from ._ext import ext, want_kernels

    if want_kernels(k, use_kernels) and scan_kernel_supported(weights, k, chunk, act):
        E = ext()
        # kernel layout: hidden index fastest, [N, 64, 256] (W1^T, S1^T, W2, S2)
        W1t = weights[0].float().transpose(1, 2).contiguous()
        S1t = momentum[0].float().transpose(1, 2).contiguous()
        W2 = weights[1].float().contiguous().clone()
        S2 = momentum[1].float().contiguous().clone()
        bf = torch.bfloat16
        y = E.memory_scan_fwd(W1t, S1t, W2, S2, k.to(bf).contiguous(), v.to(bf).contiguous(),
                              q.to(bf).contiguous(), theta.float().contiguous(), eta.float().contiguous(),
                              alpha.float().contiguous())
        return y, [W1t.transpose(1, 2), W2], [S1t.transpose(1, 2), S2]
    y, W, S, _ = memory_scan_reference(weights, momentum, k, v, q, theta, eta, alpha, chunk, act)
    return y, W, S


def head_blocks(w: torch.Tensor, heads: int) -> torch.Tensor:
    """Diagonal blocks of a ``[out, in]`` weight: ``[heads, out/heads, in/heads]``."""
    o, i = w.shape
    blocks = w.reshape(heads, o // heads, heads, i // heads)
    return torch.stack([blocks[h, :, h, :] for h in range(heads)], 0)


__all__ = ["chunk_coefficients", "memory_scan_reference", "memory_recurrence_tokenwise", "head_blocks",
           "memory_scan", "scan_kernel_supported"]
