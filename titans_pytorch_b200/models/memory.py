"""Neural long-term memory (the Titans test-time-learning memory).

Public surface follows the reference (`src/titans/memory.py:64-530`):
``MemoryState`` (weights + momentum lists, ``detach``/``clone``),
``MemoryMLP`` (``layers`` of bias-free Linears, ``get_weights``/``set_weights``/
``compute_loss``) and ``NeuralLongTermMemory`` (``proj_k/v/q``, depthwise
``conv_k/v/q``, ``memory``, ``gate_decay/lr/momentum``, ``proj_out``;
``forward(x, state, return_state)``, ``retrieve``, ``init_state``).

``semantics="ref"`` (default) reproduces the reference's CUDA behaviour,
including that ``set_weights`` writes the state into the parameters' storage
(`memory.py:162-165`), so a MAC forward leaves the last chunk's memory in the
parameters and the backward reads those values.  ``semantics="paper"`` is the
paper's per-sample, per-head memory with per-token gates and a chunked update
(:mod:`titans_pytorch_b200.ops.memory_paper`): ``memory_heads`` memories per
sample, each initialised from the diagonal block of the shared ``MemoryMLP``
weights (so the parameter layout is the reference's); per-token, per-head
gates are the head means of the sigmoid gate projections, scaled by
``memory_lr`` (theta), ``memory_momentum`` (eta) and ``memory_decay`` (alpha);
states are ``[B, heads, out, in]``.  In paper mode the outer loss trains the
query path and ``proj_out``; the memory state, keys, values and gates are
learned at test time only.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import TitansConfig
from ..ops.conv import conv_silu_norm
from ..ops.memory import (activation, activation_fn, memory_grads_reference, memory_mlp, memory_step,
                          memory_step_sharded, mlp_forward_reference, mlp_kernel_ok)
from ..ops.linear import linear
from ..ops.memory_paper import head_blocks, memory_scan, memory_scan_reference


def get_activation(name: str) -> nn.Module:
    table = {"silu": nn.SiLU, "gelu": nn.GELU, "relu": nn.ReLU}
    if name not in table:
        raise ValueError(f"Unknown activation: {name}")
    return table[name]()


@dataclass
class MemoryState:
    """Memory weights and surprise momentum carried between calls/chunks."""

    weights: list[torch.Tensor]
    momentum: list[torch.Tensor]

    def detach(self) -> "MemoryState":
        return MemoryState([w.detach() for w in self.weights], [m.detach() for m in self.momentum])

    def clone(self) -> "MemoryState":
        return MemoryState([w.clone() for w in self.weights], [m.clone() for m in self.momentum])

    def to(self, *args, **kwargs) -> "MemoryState":
        return MemoryState([w.to(*args, **kwargs) for w in self.weights],
                           [m.to(*args, **kwargs) for m in self.momentum])


class MemoryMLP(nn.Module):
    """The memory itself: L_M = 1 is one D x D matrix; L_M >= 2 is D -> H -> ... -> D."""

    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.num_layers = config.num_memory_layers
        self.dim = config.dim
        self.hidden_dim = config.memory_hidden_dim
        dims = ([self.dim, self.dim] if self.num_layers == 1 else
                [self.dim] + [self.hidden_dim] * (self.num_layers - 1) + [self.dim])
        self.layers = nn.ModuleList(nn.Linear(dims[i], dims[i + 1], bias=False)
                                    for i in range(self.num_layers))
        self.activation = get_activation(config.activation)
        for layer in self.layers:
            nn.init.normal_(layer.weight, std=config.init_std)

    def weight_list(self) -> list[torch.Tensor]:
        return [layer.weight for layer in self.layers]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # same math as mlp_forward_reference; on CUDA (bf16) one fused tcgen05
        # autograd node, else ops.linear per layer (weight gradients accumulated
        # in place under the trainer either way)
        act, uk = self.config.activation, getattr(self.config, "use_kernels", None)
        ws = self.weight_list()
        if mlp_kernel_ok(x, ws, act, uk):
            return memory_mlp(x, ws, act)
        h = x
        for i, layer in enumerate(self.layers):
            h = linear(h, layer.weight, use_kernels=uk)
            if i < self.num_layers - 1:
                h = activation(h, act, uk)
        return h

    def get_weights(self) -> list[torch.Tensor]:
        return [layer.weight.detach().clone() for layer in self.layers]

    def set_weights(self, weights: list[torch.Tensor]) -> None:
        """Write ``weights`` into the parameters' storage (not tracked by autograd)."""
        with torch.no_grad():
            for layer, w in zip(self.layers, weights, strict=True):
                if layer.weight.data.data_ptr() != w.data_ptr():
                    layer.weight.data.copy_(w)

    def compute_loss(self, keys: torch.Tensor, values: torch.Tensor) -> torch.Tensor:
        return F.mse_loss(self(keys), values, reduction="mean")


class _PaperScan(torch.autograd.Function):
    """Chunked paper-mode scan; differentiable in the queries only.

    The memory state, keys, values and gates are test-time-learned (constants
    for the outer loss).  The backward re-runs the scan to rebuild each chunk's
    start weights and back-propagates the retrieval through them.
    """

    @staticmethod
    def forward(ctx, q, k, v, theta, eta, alpha, chunk, act, use_kernels, nlayers, *state):
        W, S = list(state[:nlayers]), list(state[nlayers:])
        y, Wn, Sn = memory_scan(W, S, k, v, q.detach(), theta, eta, alpha, chunk, act, use_kernels)
        ctx.save_for_backward(q, k, v, theta, eta, alpha, *state)
        ctx.meta = (chunk, act, nlayers)
        outs = [y.to(q.dtype)] + [w.detach() for w in Wn] + [m.detach() for m in Sn]
        for t in outs[1:]:
            ctx.mark_non_differentiable(t)
        return tuple(outs)

    @staticmethod
    def backward(ctx, dy, *_):
        q, k, v, theta, eta, alpha, *state = ctx.saved_tensors
        chunk, act, nlayers = ctx.meta
        _, _, _, dq = memory_scan_reference(state[:nlayers], state[nlayers:], k, v, q, theta, eta, alpha, chunk,
                                            act, dy=dy)
        return (dq.to(q.dtype),) + (None,) * (9 + len(state))


class NeuralLongTermMemory(nn.Module):
    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.dim = config.dim
        D = config.dim
        self.use_kernels = config.use_kernels
        self.proj_k = nn.Linear(D, D, bias=False)
        self.proj_v = nn.Linear(D, D, bias=False)
        self.proj_q = nn.Linear(D, D, bias=False)
        self.use_conv = config.use_conv
        if self.use_conv:
            ks = config.conv_kernel_size
            self.conv_k = nn.Conv1d(D, D, ks, padding=ks - 1, groups=D)
            self.conv_v = nn.Conv1d(D, D, ks, padding=ks - 1, groups=D)
            self.conv_q = nn.Conv1d(D, D, ks, padding=ks - 1, groups=D)
        self.memory = MemoryMLP(config)
        self.gate_decay = nn.Sequential(nn.Linear(D, D), nn.Sigmoid())
        self.gate_lr = nn.Sequential(nn.Linear(D, D), nn.Sigmoid())
        self.gate_momentum = nn.Sequential(nn.Linear(D, D), nn.Sigmoid())
        self.proj_out = nn.Linear(D, D, bias=False)
        for m in (self.proj_k, self.proj_v, self.proj_q, self.proj_out):
            nn.init.normal_(m.weight, std=config.init_std)

    # ------------------------------------------------------------------ helpers
    def _conv(self, name: str):
        if not self.use_conv:
            return None, None
        c = getattr(self, name)
        return c.weight, c.bias

    def _gate_params(self):
        g = (self.gate_decay[0], self.gate_lr[0], self.gate_momentum[0])
        return [m.weight for m in g], [m.bias for m in g]

    # ContextShard while the owning model runs context-parallel (parallel.context)
    cp = None

    def _trim(self, x: torch.Tensor, rows: int) -> tuple[torch.Tensor, int]:
        """Keep of the ``rows`` leading halo rows of ``x`` only the ``K - 1`` the
        causal convolutions read."""
        if rows == 0:
            return x, 0
        keep = min(rows, self.config.conv_kernel_size - 1 if self.use_conv else 0)
        return x[:, rows - keep:], keep

    @staticmethod
    def _drop(t: torch.Tensor, rows: int) -> torch.Tensor:
        return t[:, rows:].contiguous() if rows else t

    def _queries(self, x: torch.Tensor, context_rows: int = 0) -> torch.Tensor:
        x, r = self._trim(x, context_rows)
        wq, bq = self._conv("conv_q")
        return self._drop(conv_silu_norm(linear(x, self.proj_q.weight, use_kernels=self.use_kernels), wq, bq,
                                         True, self.use_kernels), r)

    # per-forward cache of derived weights, set by the owning model (see SegmentedAttention)
    _wcache: dict | None = None

    @torch.no_grad()
    def _keys_values(self, x: torch.Tensor, context_rows: int = 0):
        D = self.dim
        x, r = self._trim(x, context_rows)
        kv = linear(x, self.proj_k.weight, self.proj_v.weight, use_kernels=self.use_kernels)
        wk, bk = self._conv("conv_k")
        wv, bv = self._conv("conv_v")
        k = conv_silu_norm(kv[..., :D], wk, bk, True, self.use_kernels)
        v = conv_silu_norm(kv[..., D:], wv, bv, False, self.use_kernels)
        return self._drop(k, r), self._drop(v, r)

    def _apply_conv(self, k, v, q):
        """Causal depthwise convolution of k, v, q (no activation); API parity helper."""
        from ..ops.conv import causal_dwconv_reference
        if not self.use_conv:
            return k, v, q
        return (causal_dwconv_reference(k, self.conv_k.weight, self.conv_k.bias),
                causal_dwconv_reference(v, self.conv_v.weight, self.conv_v.bias),
                causal_dwconv_reference(q, self.conv_q.weight, self.conv_q.bias))

    @property
    def _linear_silu(self) -> bool:
        """L_M = 1 without conv takes the reference's analytic SiLU gradient."""
        return self.config.num_memory_layers == 1 and not self.use_conv

    @property
    def _freezes_mlp(self) -> bool:
        """L_M = 1 with conv: the reference's fallback path leaves the MLP frozen."""
        return self.config.num_memory_layers == 1 and self.use_conv

    def _compute_gradients(self, keys: torch.Tensor, values: torch.Tensor) -> list[torch.Tensor]:
        """Associative-loss gradient at the current memory weights (ref semantics)."""
        with torch.no_grad():
            g = memory_grads_reference(keys.detach(), values.detach(),
                                       [w.detach() for w in self.memory.weight_list()],
                                       self.config.activation, self._linear_silu)
        if self._freezes_mlp:
            self.memory.requires_grad_(False)
        return g

    # -------------------------------------------------------------- paper mode
    @property
    def paper(self) -> bool:
        return self.config.semantics == "paper"

    def _heads(self) -> tuple[int, int]:
        h = self.config.memory_heads
        return h, self.dim // h

    def _split_heads(self, t: torch.Tensor) -> torch.Tensor:
        """[B, T, D] -> [B*h, T, D/h]."""
        B, T, _ = t.shape
        h, dh = self._heads()
        return t.reshape(B, T, h, dh).permute(0, 2, 1, 3).reshape(B * h, T, dh)

    def _merge_heads(self, t: torch.Tensor, B: int) -> torch.Tensor:
        h, dh = self._heads()
        T = t.shape[1]
        return t.reshape(B, h, T, dh).permute(0, 2, 1, 3).reshape(B, T, h * dh)

    def _paper_inputs(self, x: torch.Tensor):
        """Per-head unit queries (differentiable), keys, values and per-token gates."""
        D = self.dim
        h, dh = self._heads()
        B, T, _ = x.shape
        wq, bq = self._conv("conv_q")
        q = conv_silu_norm(linear(x, self.proj_q.weight, use_kernels=self.use_kernels), wq, bq, False,
                           self.use_kernels)
        q = F.normalize(self._split_heads(q), dim=-1)
        with torch.no_grad():
            kv = linear(x, self.proj_k.weight, self.proj_v.weight, use_kernels=self.use_kernels)
            wk, bk = self._conv("conv_k")
            wv, bv = self._conv("conv_v")
            k = F.normalize(self._split_heads(conv_silu_norm(kv[..., :D], wk, bk, False, self.use_kernels)), dim=-1)
            v = self._split_heads(conv_silu_norm(kv[..., D:], wv, bv, False, self.use_kernels))
            gw, gb = self._gate_params()
            g = torch.sigmoid(F.linear(x, torch.cat(gw, 0), torch.cat(gb, 0)).float())
            g = g.view(B, T, 3, h, dh).mean(-1).permute(2, 0, 3, 1).reshape(3, B * h, T)
            alpha = g[0] * self.config.memory_decay
            theta = g[1] * self.config.memory_lr
            eta = g[2] * self.config.memory_momentum
        return q, k, v, theta.contiguous(), eta.contiguous(), alpha.contiguous()

    def _paper_flat(self, state: MemoryState):
        return ([w.reshape(-1, *w.shape[-2:]) for w in state.weights],
                [m.reshape(-1, *m.shape[-2:]) for m in state.momentum])

    def _paper_scan(self, x: torch.Tensor, state: MemoryState):
        B = x.shape[0]
        h, _ = self._heads()
        q, k, v, theta, eta, alpha = self._paper_inputs(x)
        W, S = self._paper_flat(state)
        L = len(W)
        outs = _PaperScan.apply(q, k, v, theta, eta, alpha, self.config.memory_chunk_size, self.config.activation,
                                self.use_kernels, L, *W, *S)
        y = self._merge_heads(outs[0], B)
        shape = lambda t: t.reshape(B, h, *t.shape[-2:])  # noqa: E731
        return y, MemoryState([shape(w) for w in outs[1:1 + L]], [shape(m) for m in outs[1 + L:]])

    def _paper_retrieve(self, x: torch.Tensor, state: MemoryState) -> torch.Tensor:
        B = x.shape[0]
        q = self._paper_inputs(x)[0]
        W, _ = self._paper_flat(state)
        f = activation_fn(self.config.activation)
        hcur = q.float()
        for i, w in enumerate(W):
            hcur = torch.bmm(hcur, w.float().transpose(1, 2))
            if i < len(W) - 1:
                hcur = f(hcur)
        return self._merge_heads(hcur.to(x.dtype), B)

    # --------------------------------------------------------------------- API
    def init_state(self, batch_size: int = 1, device=None) -> MemoryState:
        if self.paper:
            h, _ = self._heads()
            w = [head_blocks(t.detach().float(), h) for t in self.memory.weight_list()]
            w = [t.unsqueeze(0).expand(batch_size, *t.shape).clone() for t in w]
            if device is not None:
                w = [t.to(device) for t in w]
            return MemoryState(weights=w, momentum=[torch.zeros_like(t) for t in w])
        w = self.memory.get_weights()
        return MemoryState(weights=w, momentum=[torch.zeros_like(t) for t in w])

    def _update(self, x: torch.Tensor, state: MemoryState, context_rows: int = 0) -> MemoryState:
        """New state after one update with the tokens of ``x`` (no retrieval output).

        ``context_rows`` leading rows of ``x`` are a halo from the previous
        sequence shard: read by the convolutions only.  Under context
        parallelism the update averages its statistics over the shards.
        """
        if self.paper:
            with torch.no_grad():
                return self._paper_scan(x.detach(), state)[1]
        k, v = self._keys_values(x, context_rows)
        gw, gb = self._gate_params()
        xs = x[:, context_rows:].detach()
        if self.cp is not None and self.cp.active:
            new_w, new_m = memory_step_sharded(k, v, xs, state.weights, state.momentum, gw, gb,
                                               self.config.memory_lr, self.config.memory_momentum,
                                               self.config.activation, self._linear_silu, self.use_kernels,
                                               self.cp)
        else:
            new_w, new_m = memory_step(k, v, xs, state.weights, state.momentum, gw, gb,
                                       self.config.memory_lr, self.config.memory_momentum,
                                       self.config.activation, self._linear_silu, self.use_kernels)
        if self._freezes_mlp:
            self.memory.requires_grad_(False)
        return MemoryState(new_w, new_m).detach()

    def forward(self, x: torch.Tensor, state: MemoryState | None = None,
                return_state: bool = True, update: bool = True, context_rows: int = 0):
        """Retrieve with the incoming memory and update it with ``x``.

        The first ``context_rows`` rows of ``x`` are a halo from the previous
        sequence shard (context parallelism): they feed the convolutions and
        produce no output row.

        Returns ``(proj_out(M_{t-1}(q)), new_state or None)``.  ``update=False``
        skips the (gradient-free) update and returns no state; activation
        checkpointing uses it to run the update once, outside the recomputed
        region.
        """
        if state is None:
            state = self.init_state(x.shape[0], x.device)
        elif not self.paper:
            self.memory.set_weights(state.weights)
        if self.paper:
            if context_rows:
                raise NotImplementedError("paper semantics has no context-parallel form")
            y, new_state = self._paper_scan(x, state)
            out = F.linear(y, self.proj_out.weight)
            return (out, new_state) if return_state else (out, None)
        retrieved = self.memory(self._queries(x, context_rows))
        new_state = self._update(x, state, context_rows) if update else None
        out = linear(retrieved, self.proj_out.weight, use_kernels=self.use_kernels)
        return (out, new_state) if return_state else (out, None)

    def retrieve(self, queries: torch.Tensor, state: MemoryState) -> torch.Tensor:
        """proj_out(M(q)) with the memory set to ``state`` (no update)."""
        if self.paper:
            return F.linear(self._paper_retrieve(queries, state), self.proj_out.weight)
        self.memory.set_weights(state.weights)
        return linear(self.memory(self._queries(queries)), self.proj_out.weight, use_kernels=self.use_kernels)


__all__ = ["MemoryState", "MemoryMLP", "NeuralLongTermMemory", "get_activation", "activation_fn"]
