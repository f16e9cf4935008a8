"""Incremental (token-by-token) decoding with a sliding-window KV ring cache and
carried memory state, for MAG, MAL and LMM (reference semantics).

The reference decodes by re-running the model on the last ``chunk_size``
tokens for every new token, updating the memory on every call
(`scripts/inference.py:321-423`); its ``StaticKVCache``
(`src/titans/optimized_inference.py:46-135`) is never wired into the
models.  :func:`~titans_pytorch_b200.inference.generate.generate` keeps that
recurrence.  This module is the streaming alternative: one token per step at
O(window) attention and O(1) memory cost.

Streaming semantics (what one step computes, per block):

* attention: the token's query (RoPE at its stream position ``P + t``) over
  the persistent tokens' keys (positions ``0..P-1``) and the keys of the last
  ``window`` tokens of the stream, kept rotated in a ring of ``window`` slots
  per layer (slot ``t mod window``);
* memory retrieval: ``proj_out(M_state(q_t))`` with ``q_t`` the causal
  depthwise conv (ring of the last ``K - 1`` projected queries) + SiLU + L2
  of the projected query, and ``M_state`` the memory MLP at the carried state;
* memory update: every ``update_every`` tokens (default ``chunk_size``) the
  memory inputs of those tokens go through the block's own update
  (``NeuralLongTermMemory._update``), exactly as a forward call over those
  tokens would update it, and the new state is carried.

Until the first update this equals a full forward over the stream's prefix
(per-token logits of ``model(ids[:, :t+1])``), and the state after the first
``update_every`` tokens equals ``model(ids[:, :update_every])``'s new state;
the tests check both, and the ring's wrap-around past ``window`` tokens.
"""

from __future__ import annotations

import torch

from ..models.memory import MemoryState
from ..ops.attention import rope_angles
from ..ops.conv import conv_silu_norm_reference
from ..ops.linear import linear
from ..ops.memory import activation


def _rotate(x: torch.Tensor, pos: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair RoPE of ``x`` [B, S, H, d] at positions ``pos`` [S] (fp32 math)."""
    cos, sin = rope_angles(pos, inv_freq)
    cos, sin = cos[None, :, None, :], sin[None, :, None, :]
    xf = x.float()
    x1, x2 = xf[..., 0::2], xf[..., 1::2]
    out = torch.empty_like(xf)
    out[..., 0::2] = x1 * cos - x2 * sin
    out[..., 1::2] = x1 * sin + x2 * cos
    return out


class _LayerCache:
    """Per-block decode state: K/V ring, persistent keys, query-conv ring, the
    memory inputs of the current update interval, and the memory state (all
    updated in place, so a captured step replays on the same buffers)."""

    def __init__(self, block, batch: int, window: int, interval: int, device, dtype, state) -> None:
        self.block = block
        att = getattr(block, "attention", None)
        self.att = att
        mem = block.memory
        D = mem.dim
        self.P = 0
        if att is not None:
            H, d = att.num_heads, att.head_dim
            self.k = torch.zeros(batch, window, H, d, dtype=torch.float32, device=device)
            self.v = torch.zeros(batch, window, H, d, dtype=torch.float32, device=device)
            pers = block.persistent(1)
            P = pers.shape[1] if pers is not None else 0
            self.P = P
            if P:
                pkv = att._project(pers[:1], kv_only=True)
                pk = pkv[..., :D].reshape(1, P, H, d)
                pv = pkv[..., D:].reshape(1, P, H, d).float()
                if att.rope is not None:
                    pk = _rotate(pk, torch.arange(P, device=device), att.rope.inv_freq)
                self.pk = pk.float().expand(batch, -1, -1, -1).contiguous()
                self.pv = pv.expand(batch, -1, -1, -1).contiguous()
        ks = mem.config.conv_kernel_size if mem.use_conv else 1
        self.qring = torch.zeros(batch, max(ks - 1, 0), D, dtype=dtype, device=device)
        self.pending = torch.zeros(batch, interval, D, dtype=dtype, device=device)
        st = state if state is not None else mem.init_state(batch, device)
        self.state = MemoryState([w.clone() for w in st.weights], [m.clone() for m in st.momentum])


class StreamingDecoder:
    """Token-by-token decoder; see the module docstring.

    ``step(tokens [B, 1]) -> logits [B, V]``; ``states`` exposes the carried
    memory states (one :class:`MemoryState` per block).  ``graph=True``
    (CUDA) captures the per-token step once and replays it (the step is a few
    hundred small launches); the memory update between intervals runs
    eagerly and writes the states in place."""

    def __init__(self, model, batch: int = 1, window: int | None = None, update_every: int | None = None,
                 states=None, graph: bool = False) -> None:
        cfg = model.config
        if getattr(model, "model_type", "") == "mac":
            raise NotImplementedError("incremental decoding covers MAG, MAL and LMM; MAC attends over memory "
                                      "tokens retrieved for the whole segment (use generate())")
        if cfg.semantics != "ref":
            raise NotImplementedError("incremental decoding runs the reference semantics")
        self.model = model
        self.kind = model.model_type
        p = next(model.parameters())
        self.device, self.dtype = p.device, p.dtype
        self.window = int(window or cfg.window_size)
        self.update_every = int(update_every or cfg.chunk_size)
        self.batch = batch
        sts = states if states is not None else [None] * len(model.blocks)
        with torch.no_grad():
            self.layers = [_LayerCache(b, batch, self.window, self.update_every, self.device, self.dtype, st)
                           for b, st in zip(model.blocks, sts, strict=True)]
        self.t = 0                                                          # host copy
        self.t_dev = torch.zeros(1, dtype=torch.long, device=self.device)   # the step's position
        self.ring_pos = torch.arange(self.window, device=self.device)
        self.graph = bool(graph) and self.device.type == "cuda"
        self._graph = None
        self._tok = torch.zeros(batch, 1, dtype=torch.long, device=self.device)
        self._logits = None

    @property
    def states(self) -> list[MemoryState]:
        return [lc.state for lc in self.layers]

    # ------------------------------------------------------------ pieces
    def _attend(self, lc: _LayerCache, n: torch.Tensor) -> torch.Tensor:
        att = lc.att
        B = n.shape[0]
        H, d = att.num_heads, att.head_dim
        D = H * d
        qkv = att._project(n)  # [B, 1, 3D]
        q = qkv[..., :D].reshape(B, 1, H, d)
        k = qkv[..., D:2 * D].reshape(B, 1, H, d)
        v = qkv[..., 2 * D:].reshape(B, 1, H, d)
        if att.rope is not None:
            pos = self.t_dev + lc.P
            q = _rotate(q, pos, att.rope.inv_freq)
            k = _rotate(k, pos, att.rope.inv_freq)
        slot = self.t_dev % self.window
        lc.k.index_copy_(1, slot, k.float())
        lc.v.index_copy_(1, slot, v.float())
        s = torch.einsum("bhd,bshd->bhs", q[:, 0].float(), lc.k) * att.scale
        # ring slot j holds a token once the stream has passed it (all slots after the first wrap)
        s = s.masked_fill((self.ring_pos > self.t_dev)[None, None, :], float("-inf"))
        if lc.P:
            sp = torch.einsum("bhd,bshd->bhs", q[:, 0].float(), lc.pk) * att.scale
            pr = torch.softmax(torch.cat([sp, s], dim=-1), dim=-1)
            o = torch.einsum("bhs,bshd->bhd", pr[..., :lc.P], lc.pv) + \
                torch.einsum("bhs,bshd->bhd", pr[..., lc.P:], lc.v)
        else:
            o = torch.einsum("bhs,bshd->bhd", torch.softmax(s, dim=-1), lc.v)
        o = o.reshape(B, 1, D).to(n.dtype)
        return linear(o, att.proj_out.weight, use_kernels=att.use_kernels)

    def _retrieve(self, lc: _LayerCache, n: torch.Tensor) -> torch.Tensor:
        mem = lc.block.memory
        qp = linear(n, mem.proj_q.weight, use_kernels=mem.use_kernels)  # [B, 1, D]
        if mem.use_conv:
            win = torch.cat([lc.qring, qp], dim=1)  # the last K projected queries
            q = conv_silu_norm_reference(win.float(), mem.conv_q.weight.float(), mem.conv_q.bias.float(),
                                         True)[:, -1:].to(n.dtype)
            if lc.qring.shape[1]:
                lc.qring.copy_(win[:, 1:])
        else:
            q = conv_silu_norm_reference(qp.float(), None, None, True).to(n.dtype)
        # the memory MLP at the carried state (the forward writes the state into the MLP's
        # weights first; reading the state tensors directly gives the same product)
        h = q
        ws = lc.state.weights
        for i, w in enumerate(ws):
            h = linear(h, w.to(n.dtype), use_kernels=mem.use_kernels)
            if i < len(ws) - 1:
                h = activation(h, mem.config.activation, mem.use_kernels)
        return linear(h, mem.proj_out.weight, use_kernels=mem.use_kernels)

    def _block(self, lc: _LayerCache, x: torch.Tensor) -> torch.Tensor:
        from ..models.titans import _ffn_residual

        blk = lc.block
        n = blk.norm1(x)
        lc.pending.index_copy_(1, self.t_dev % self.update_every, n)
        if self.kind == "mag":
            y = x + self._attend(lc, n)
            out = y * self._retrieve(lc, n)
            return _ffn_residual(blk, out, blk.norm2(out))
        m = self._retrieve(lc, n)
        x, n2 = blk.norm2.forward_with_residual(x, m)
        if self.kind == "mal":
            x, n3 = blk.norm3.forward_with_residual(x, self._attend(lc, n2))
            return _ffn_residual(blk, x, n3)
        return _ffn_residual(blk, x, n2)

    def _core(self, tokens: torch.Tensor) -> torch.Tensor:
        model = self.model
        x = model.embed(tokens)
        for lc in self.layers:
            x = self._block(lc, x)
        logits = linear(model.norm(x), model.head.weight, use_kernels=model.config.use_kernels)[:, -1]
        self.t_dev += 1
        return logits

    # ------------------------------------------------------------ API
    @torch.no_grad()
    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """Logits [B, V] of the next token after ``tokens`` [B, 1] (with ``graph``,
        the returned tensor is overwritten by the next step)."""
        tokens = tokens.to(self.device)
        if not self.graph:
            logits = self._core(tokens)
        elif self._graph is None and self.t == 0:
            # the first step runs eagerly on a side stream (it also warms the libraries up)
            cur = torch.cuda.current_stream(self.device)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                logits = self._core(tokens)
            cur.wait_stream(side)
        else:
            if self._graph is None:
                g = torch.cuda.CUDAGraph()
                self._tok.copy_(tokens)
                with torch.cuda.graph(g):
                    self._logits = self._core(self._tok)
                self._graph = g
            self._tok.copy_(tokens)
            self._graph.replay()
            logits = self._logits
        self.t += 1
        if self.t % self.update_every == 0:
            self._update_memory()
        return logits

    def _update_memory(self) -> None:
        for lc in self.layers:
            new = lc.block.memory._update(lc.pending, lc.state)
            for a, b in zip(lc.state.weights + lc.state.momentum, new.weights + new.momentum, strict=True):
                a.copy_(b)

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Feed a prompt [B, T] token by token; returns the last logits [B, V]."""
        logits = None
        for i in range(input_ids.shape[1]):
            logits = self.step(input_ids[:, i:i + 1])
        return logits


@torch.no_grad()
def generate_incremental(model, input_ids: torch.Tensor, max_new_tokens: int = 100, temperature: float = 1.0,
                         top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.0,
                         eos_token_id: int | None = None, greedy: bool = False,
                         generator: torch.Generator | None = None, window: int | None = None,
                         update_every: int | None = None):
    """Generate with :class:`StreamingDecoder`; returns ``(ids, states)``."""
    from .generate import sample_next

    dec = StreamingDecoder(model, batch=input_ids.shape[0], window=window, update_every=update_every,
                           graph=input_ids.is_cuda)
    logits = dec.prefill(input_ids)
    generated = input_ids.to(dec.device).clone()
    for _ in range(max_new_tokens):
        nxt = sample_next(logits.clone(), generated, temperature, top_k, top_p, repetition_penalty, greedy, generator)
        generated = torch.cat([generated, nxt.to(generated.dtype)], dim=1)
        if eos_token_id is not None and bool((nxt == eos_token_id).all()):
            break
        logits = dec.step(nxt)
    return generated, dec.states


__all__ = ["StreamingDecoder", "generate_incremental"]
