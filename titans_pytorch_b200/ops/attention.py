"""Windowed causal attention with always-visible prefix keys and fused RoPE.

One op serves both attention forms of the reference:

* sliding-window attention (`src/titans/attention.py:135-307`): queries come
  from ``x`` only, keys/values from ``[prefix || x]``; a query at main
  position i sees every prefix key and main keys j with ``j <= i`` and
  ``i - j < window``.  RoPE positions are ``P + i`` for queries, ``p`` for
  prefix keys and ``P + j`` for main keys (`attention.py:248-251`).
* MAC segmented attention (`attention.py:355-424`): causal attention over
  ``[persistent || memory || x]`` whose output is kept only for the ``x``
  rows.  Those rows see the whole prefix and causal main keys, i.e. the same
  rule with an infinite window, so the discarded prefix query rows are never
  computed.

``pos_offset`` shifts the RoPE positions of the main rows (queries and main
keys) to ``P + pos_offset + i`` while prefix keys keep ``0..P-1``: a sequence
shard that starts at global token ``pos_offset`` then attends exactly as the
same rows of the whole sequence would.

RoPE is the interleaved-pair rotation of the reference (`attention.py:107-132`),
base 10000, applied on load inside the CUDA kernel (``csrc/attention.cu``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext, want_kernels

NO_WINDOW = 1 << 30


def rope_angles(positions: torch.Tensor, inv_freq: torch.Tensor):
    freqs = torch.outer(positions.float(), inv_freq.float())
    return freqs.cos(), freqs.sin()


def apply_rope_reference(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (x[..., 2i], x[..., 2i+1]) of ``x`` [B, S, H, d]."""
    cos = cos.to(x.dtype)[None, :, None, :]
    sin = sin.to(x.dtype)[None, :, None, :]
    x1, x2 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x1 * cos - x2 * sin
    out[..., 1::2] = x1 * sin + x2 * cos
    return out


def prefix_window_mask(q_len: int, prefix_len: int, window: int, device) -> torch.Tensor:
    """Boolean [q_len, prefix_len + q_len] mask (True = attend)."""
    i = torch.arange(q_len, device=device)[:, None]
    j = torch.arange(q_len, device=device)[None, :]
    main = (j <= i) & ((i - j) < window)
    pre = torch.ones(q_len, prefix_len, dtype=torch.bool, device=device)
    return torch.cat([pre, main], dim=1)


def _split_qkv(qkv, pkv, H):
    B, T, D3 = qkv.shape
    D = D3 // 3
    d = D // H
    q, k, v = (qkv[..., i * D:(i + 1) * D].reshape(B, T, H, d) for i in range(3))
    pk = pv = None
    if pkv is not None and pkv.shape[1] > 0:
        pk = pkv[..., :D].reshape(pkv.shape[0], pkv.shape[1], H, d)
        pv = pkv[..., D:].reshape(pkv.shape[0], pkv.shape[1], H, d)
    return q, k, v, pk, pv


def window_attention_reference(qkv, pkv, H, window, scale, inv_freq, dropout_p=0.0, training=False,
                               pos_offset=0):
    """PyTorch restatement (dense mask + SDPA).  Returns [B, T, H, d]."""
    q, k, v, pk, pv = _split_qkv(qkv, pkv, H)
    B, T, _, d = q.shape
    P = 0 if pk is None else pk.shape[1]
    if P:
        kf = torch.cat([pk.expand(B, -1, -1, -1), k], dim=1)
        vf = torch.cat([pv.expand(B, -1, -1, -1), v], dim=1)
    else:
        kf, vf = k, v
    if inv_freq is not None:
        main = torch.arange(P, P + T, device=q.device) + pos_offset
        cq, sq = rope_angles(main, inv_freq)
        ck, sk = rope_angles(torch.cat([torch.arange(0, P, device=q.device), main]), inv_freq)
        q = apply_rope_reference(q, cq, sq)
        kf = apply_rope_reference(kf, ck, sk)
    mask = prefix_window_mask(T, P, window, q.device)
    add = torch.zeros(mask.shape, dtype=q.dtype, device=q.device).masked_fill_(~mask, float("-inf"))
    o = F.scaled_dot_product_attention(
        q.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2), attn_mask=add,
        dropout_p=dropout_p if training else 0.0, is_causal=False, scale=scale)
    return o.transpose(1, 2)


class _WindowAttnFn(torch.autograd.Function):
    """pack (RoPE + head-major layout) -> flash forward; backward -> unpack."""

    @staticmethod
    def forward(ctx, qkv, pkv, H, window, scale, inv_freq, pos_offset):
        E = ext()
        Q, K, V = E.attn_pack(qkv, pkv, H, inv_freq, pos_offset)
        if E.attn_tc_fwd_supported(Q.shape[-1]):
            O, lse = E.attn_fwd_tc(Q, K, V, window, scale)      # tcgen05 / TMEM / TMA (head_dim 64, 96)
        else:
            O, lse = E.attn_fwd_packed(Q, K, V, window, scale)  # mma.sync path (other head dims)
        ctx.save_for_backward(Q, K, V, O, lse, inv_freq)
        ctx.window, ctx.scale, ctx.pos_offset = window, scale, pos_offset
        ctx.bp = 0 if pkv is None else pkv.shape[0]
        ctx.dtype = qkv.dtype
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, lse, inv_freq = ctx.saved_tensors
        E = ext()
        if E.attn_tc_supported(Q.shape[-1]):
            dQa, dKa, dVa = E.attn_bwd_tc(dO, Q, K, V, O, lse, ctx.window, ctx.scale)      # tcgen05
        else:
            dQa, dKa, dVa = E.attn_bwd_packed(dO, Q, K, V, O, lse, ctx.window, ctx.scale)  # mma.sync
        dqkv, dpkv = E.attn_unpack(dQa, dKa, dVa, inv_freq, max(ctx.bp, 1), ctx.dtype, ctx.pos_offset)
        return dqkv, (dpkv if ctx.bp else None), None, None, None, None, None


def window_attention(qkv: torch.Tensor, pkv: torch.Tensor | None, num_heads: int,
                     window: int | None = None, scale: float | None = None,
                     inv_freq: torch.Tensor | None = None, dropout_p: float = 0.0,
                     training: bool = False, use_kernels: bool | None = None,
                     pos_offset: int = 0) -> torch.Tensor:
    """Attention of the queries in ``qkv`` over ``[prefix || main]`` keys.

    ``qkv`` is the fused projection ``[B, T, 3D]`` (q | k | v, last dim
    contiguous); ``pkv`` the projected prefix ``[B or 1, P, 2D]`` (k | v) or
    ``None``.  ``window=None`` means no window (MAC).  ``pos_offset`` is the
    global index of the first main row (RoPE only).  Returns ``[B, T, H, d]``.
    """
    window = NO_WINDOW if window is None else int(window)
    H = int(num_heads)
    d = qkv.shape[-1] // 3 // H
    scale = (d ** -0.5) if scale is None else float(scale)
    if pkv is not None and pkv.shape[1] == 0:
        pkv = None
    if want_kernels(qkv, use_kernels):
        if dropout_p > 0.0 and training:
            raise NotImplementedError("attention-probability dropout is not implemented in the "
                                      "sm_100a attention kernel; set dropout=0")
        return _WindowAttnFn.apply(qkv, pkv, H, window, scale, inv_freq, int(pos_offset))
    return window_attention_reference(qkv, pkv, H, window, scale, inv_freq, dropout_p, training,
                                      int(pos_offset))


def attention_flops(B: int, T: int, H: int, d: int, P: int, window: int | None) -> float:
    """Forward FLOPs actually needed (visible keys only): 4 * d per (query, key) pair."""
    w = T if window is None else min(window, T)
    # main keys: sum_i min(i+1, w)
    main = w * (w + 1) / 2 + max(T - w, 0) * w
    return 4.0 * d * H * B * (main + P * T)


__all__ = ["window_attention", "window_attention_reference", "apply_rope_reference",
           "rope_angles", "prefix_window_mask", "attention_flops", "NO_WINDOW"]
