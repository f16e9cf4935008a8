"""Attention modules: RoPE, sliding-window attention (MAG/MAL), segmented attention (MAC).

Public surface and parameter names follow the reference
(`src/titans/attention.py:23-441`): ``proj_q/k/v/out`` (no bias, N(0, init_std)),
``rope.inv_freq`` (persistent buffer).  The compute is one kernel,
:func:`titans_pytorch_b200.ops.attention.window_attention`, which replaces the
reference's dense additive mask + SDPA with a windowed flash kernel that skips
masked tiles, applies RoPE on load, and for MAC never computes the prefix
query rows whose outputs the reference discards (`attention.py:424`).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import TitansConfig
from ..ops.linear import linear
from ..ops.attention import prefix_window_mask, window_attention


class RotaryPositionEmbedding(nn.Module):
    """Interleaved-pair rotary embedding, base 10000 (RoFormer)."""

    def __init__(self, dim: int, max_seq_len: int = 8192, base: float = 10000.0) -> None:
        super().__init__()
        self.dim = dim
        self.max_seq_len = max_seq_len
        self.base = base
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self._build_cache(max_seq_len)

    def _build_cache(self, seq_len: int, device=None, dtype=None) -> None:
        inv = self.inv_freq if device is None else self.inv_freq.to(device)
        ang = torch.outer(torch.arange(seq_len, device=inv.device, dtype=torch.float32), inv.float())
        cos, sin = ang.cos(), ang.sin()
        if dtype is not None:
            cos, sin = cos.to(dtype), sin.to(dtype)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)
        self._cache_key = (device, dtype)

    def forward(self, q: torch.Tensor, k: torch.Tensor, seq_offset: int = 0):
        """Rotate ``q`` and ``k`` ([B, H, S, d]) at positions seq_offset.. ."""
        n = q.shape[2]
        if (seq_offset + n > self.cos_cached.shape[0]
                or self._cache_key != (q.device, q.dtype)):
            self._build_cache(max(seq_offset + n, self.max_seq_len), q.device, q.dtype)
        cos = self.cos_cached[seq_offset:seq_offset + n]
        sin = self.sin_cached[seq_offset:seq_offset + n]
        return self._apply_rotary(q, cos, sin), self._apply_rotary(k, cos, sin)

    @staticmethod
    def _apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        a, b = x[..., 0::2], x[..., 1::2]
        c, s = cos[None, None], sin[None, None]
        return torch.stack([a * c - b * s, a * s + b * c], dim=-1).flatten(-2)


class _AttentionBase(nn.Module):
    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.dim = config.dim
        self.num_heads = config.num_heads
        self.head_dim = config.head_dim
        self.scale = self.head_dim ** -0.5
        self.use_kernels = config.use_kernels
        self.proj_q = nn.Linear(config.dim, config.dim, bias=False)
        self.proj_k = nn.Linear(config.dim, config.dim, bias=False)
        self.proj_v = nn.Linear(config.dim, config.dim, bias=False)
        self.proj_out = nn.Linear(config.dim, config.dim, bias=False)
        self.rope: RotaryPositionEmbedding | None = None
        if config.use_rope:
            self.rope = RotaryPositionEmbedding(config.head_dim, config.max_seq_len)
        self.dropout = nn.Dropout(config.dropout)
        for m in (self.proj_q, self.proj_k, self.proj_v, self.proj_out):
            nn.init.normal_(m.weight, std=config.init_std)

    # Set by the owning model (a per-forward cache of derived weights); the
    # stacked projections below read adjacent weights in place, so nothing is cached.
    _wcache: dict | None = None

    def _attend(self, qkv, pkv, window, context_rows: int = 0, pos_offset: int = 0):
        """qkv: [B, T, 3D]; pkv: [B or 1, P, 2D] or None -> [B, T - context_rows, D] after proj_out."""
        o = window_attention(
            qkv, pkv, self.num_heads, window=window, scale=self.scale,
            inv_freq=None if self.rope is None else self.rope.inv_freq,
            dropout_p=self.dropout.p, training=self.training, use_kernels=self.use_kernels,
            pos_offset=pos_offset)
        o = o.reshape(*qkv.shape[:-1], self.dim)
        if context_rows:
            o = o[:, context_rows:].contiguous()
        return linear(o, self.proj_out.weight, use_kernels=self.use_kernels)

    def _project(self, x: torch.Tensor, kv_only: bool = False) -> torch.Tensor:
        """x @ [Wq; Wk; Wv]^T (or [Wk; Wv] with ``kv_only``); weight gradients
        accumulate in place under the trainer (see ``ops.linear``)."""
        ws = (self.proj_k.weight, self.proj_v.weight) if kv_only else (
            self.proj_q.weight, self.proj_k.weight, self.proj_v.weight)
        return linear(x, *ws, use_kernels=self.use_kernels)


class SlidingWindowAttention(_AttentionBase):
    """Causal sliding-window attention with an always-visible prefix (MAG/MAL core)."""

    def __init__(self, config: TitansConfig) -> None:
        super().__init__(config)
        self.window_size = config.window_size

    def forward(self, x: torch.Tensor, prefix: torch.Tensor | None = None,
                seq_offset: int = 0, context_rows: int = 0, position_offset: int = 0) -> torch.Tensor:
        """``x`` [B, T, D], ``prefix`` [B, P, D] or None.

        ``seq_offset`` shifts every RoPE position by the same amount; rotary
        scores depend only on position differences, so the output does not
        change with it (the argument is kept for API compatibility).

        Context parallelism: the first ``context_rows`` rows of ``x`` are the
        previous shard's last rows (keys and values only; no output row), and
        ``position_offset`` is the global token index of ``x``'s first row, so
        the prefix keys keep positions ``0..P-1`` and the shard's rows get
        their positions in the whole sequence.
        """
        del seq_offset
        qkv = self._project(x)
        pkv = None
        if prefix is not None and prefix.shape[1] > 0:
            if prefix.stride(0) == 0:  # batch-broadcast persistent tokens: project once
                prefix = prefix[:1]
            pkv = self._project(prefix, kv_only=True)
        return self._attend(qkv, pkv, self.window_size, context_rows, position_offset)

    # Mask helpers (same contract as the reference's, used by tests and debugging)
    def _create_sliding_window_mask(self, seq_len: int, device) -> torch.Tensor:
        return prefix_window_mask(seq_len, 0, self.window_size, device)

    def _create_extended_mask(self, query_len: int, key_len: int, prefix_len: int, device) -> torch.Tensor:
        assert key_len == prefix_len + query_len or key_len == prefix_len
        if key_len == prefix_len:
            m = torch.ones(query_len, prefix_len, dtype=torch.bool, device=device)
        else:
            m = prefix_window_mask(query_len, prefix_len, self.window_size, device)
        return m[None, None]


class SegmentedAttention(_AttentionBase):
    """Causal attention over ``[persistent || memory || x]``; returns the ``x`` rows (MAC core)."""

    def forward(self, x: torch.Tensor, persistent: torch.Tensor | None = None,
                memory: torch.Tensor | None = None) -> torch.Tensor:
        B = x.shape[0]
        qkv = self._project(x)
        parts = [p for p in (persistent, memory) if p is not None and p.shape[1] > 0]
        pkv = None
        if len(parts) == 1:
            pre = parts[0][:1] if parts[0].stride(0) == 0 else parts[0]
            pkv = self._project(pre, kv_only=True)
        elif len(parts) == 2:
            if persistent.stride(0) == 0:
                # shared persistent rows: project once, then broadcast over the batch
                pkv_p = self._project(persistent[:1], kv_only=True).expand(B, -1, -1)
            else:
                pkv_p = self._project(persistent, kv_only=True)
            pkv = torch.cat([pkv_p, self._project(memory, kv_only=True)], dim=1)
        return self._attend(qkv, pkv, None)

    def _create_causal_mask(self, seq_len: int, device) -> torch.Tensor:
        return torch.tril(torch.ones(seq_len, seq_len, dtype=torch.bool, device=device))[None, None]
