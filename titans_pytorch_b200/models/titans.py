"""Titans model variants: MAC (memory as context), MAG (as gate), MAL (as layer), LMM.

Block structure, parameter names and ``forward(input_ids, states=None) ->
(logits, states)`` follow the reference (`src/titans/models.py:144-737`):

* MAC (`:144-323`): per ``chunk_size`` segment, every block retrieves from its
  memory, attends over ``[persistent || norm(retrieved) || x]``, updates its
  memory with the attention output ``y`` and gates ``y * retrieve(y)``; chunks
  are the outer loop, blocks the inner loop.
* MAG (`:331-473`): ``y = x + SWA(norm1 x)``; ``o = y * Mem(norm1 x)``; FFN.
* MAL (`:481-615`): ``x += Mem(norm1 x)``; ``x += SWA(norm2 x)``; FFN.
* LMM (`:623-737`): ``x += Mem(norm1 x)``; FFN.

All four tie ``head.weight`` to ``embed.weight`` and initialise the embedding
with N(0, init_std).  Submodule registration order matches the reference so
``state_dict`` keys come out in the same order.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import TitansConfig
from ..ops.linear import linear
from .attention import SegmentedAttention, SlidingWindowAttention
from .layers import FeedForward, RMSNorm
from .memory import MemoryState, NeuralLongTermMemory
from .persistent import PersistentMemory


def _norm(config: TitansConfig) -> RMSNorm:
    return RMSNorm(config.dim, config.norm_eps, config.use_kernels)


def _halo(block: nn.Module, n: torch.Tensor, rows: int) -> tuple[torch.Tensor, int, int]:
    """Under context parallelism: ``n`` with the previous shard's last ``rows``
    rows prepended, their count, and the global index of the first row."""
    cp = getattr(block, "cp", None)
    if cp is None or not cp.active:
        return n, 0, 0
    ne, h = cp.extend(n, rows)
    return ne, h, cp.start(n.shape[1]) - h


def _conv_halo(config: TitansConfig) -> int:
    return config.conv_kernel_size - 1 if config.use_conv else 0


def _ffn_residual(block: nn.Module, x: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """``x + dropout(ffn(h))``; the add runs in the FFN's last GEMM when dropout is off."""
    if block.dropout.p == 0.0 or not block.training:
        return block.ffn(h, residual=x)
    return x + block.dropout(block.ffn(h))


class MACBlock(nn.Module):
    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.memory = NeuralLongTermMemory(config)
        self.persistent = PersistentMemory(config)
        self.attention = SegmentedAttention(config)
        self.ffn = FeedForward(config)
        self.norm1 = _norm(config)
        self.norm2 = _norm(config)
        self.norm_mem = _norm(config)
        self.dropout = nn.Dropout(config.dropout)

    def forward(self, x: torch.Tensor, state: MemoryState | None = None):
        B = x.shape[0]
        if state is None:
            state = self.memory.init_state(B, x.device)
        h = self.norm_mem(self.memory.retrieve(x, state))
        attn = self.attention(self.norm1(x), persistent=self.persistent(B), memory=h)
        y = x + self.dropout(attn)
        # The reference calls memory(y, state) here and discards its retrieval
        # output; only the updated state is used, so only the update runs.
        new_state = self.memory._update(y, state)
        out = y * self.memory.retrieve(y, new_state)
        return _ffn_residual(self, out, self.norm2(out)), new_state


class MAGBlock(nn.Module):
    cp = None  # ContextShard under context parallelism (parallel.context)

    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.persistent = PersistentMemory(config)
        self.attention = SlidingWindowAttention(config)
        self.memory = NeuralLongTermMemory(config)
        self.ffn = FeedForward(config)
        self.norm1 = _norm(config)
        self.norm2 = _norm(config)
        self.dropout = nn.Dropout(config.dropout)

    def memory_input(self, x: torch.Tensor) -> torch.Tensor:
        """The tensor the memory reads (and is updated with) for block input ``x``."""
        return self.norm1(x)

    def forward(self, x: torch.Tensor, state: MemoryState | None = None, update_memory: bool = True):
        n = self.norm1(x)
        # one halo serves the window (w - 1 rows) and the memory convolutions (K - 1)
        ne, h, pos = _halo(self, n, max(self.config.window_size - 1, _conv_halo(self.config)))
        y = x + self.dropout(self.attention(ne, prefix=self.persistent(x.shape[0]), context_rows=h,
                                            position_offset=pos))
        m, new_state = self.memory(ne, state=state, update=update_memory, context_rows=h)
        out = y * m
        return _ffn_residual(self, out, self.norm2(out)), new_state


class MALBlock(nn.Module):
    cp = None

    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.persistent = PersistentMemory(config)
        self.memory = NeuralLongTermMemory(config)
        self.attention = SlidingWindowAttention(config)
        self.ffn = FeedForward(config)
        self.norm1 = _norm(config)
        self.norm2 = _norm(config)
        self.norm3 = _norm(config)
        self.dropout = nn.Dropout(config.dropout)

    def memory_input(self, x: torch.Tensor) -> torch.Tensor:
        return self.norm1(x)

    def forward(self, x: torch.Tensor, state: MemoryState | None = None, update_memory: bool = True):
        n1, h1, _ = _halo(self, self.norm1(x), _conv_halo(self.config))
        m, new_state = self.memory(n1, state=state, update=update_memory, context_rows=h1)
        x, n2 = self.norm2.forward_with_residual(x, self.dropout(m))  # residual add fused with the norm
        n2, h2, pos = _halo(self, n2, self.config.window_size - 1)
        a = self.attention(n2, prefix=self.persistent(x.shape[0]), context_rows=h2, position_offset=pos)
        x, n3 = self.norm3.forward_with_residual(x, self.dropout(a))
        return _ffn_residual(self, x, n3), new_state


class LMMBlock(nn.Module):
    cp = None

    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.memory = NeuralLongTermMemory(config)
        self.ffn = FeedForward(config)
        self.norm1 = _norm(config)
        self.norm2 = _norm(config)
        self.dropout = nn.Dropout(config.dropout)

    def memory_input(self, x: torch.Tensor) -> torch.Tensor:
        return self.norm1(x)

    def forward(self, x: torch.Tensor, state: MemoryState | None = None, update_memory: bool = True):
        n1, h1, _ = _halo(self, self.norm1(x), _conv_halo(self.config))
        m, new_state = self.memory(n1, state=state, update=update_memory, context_rows=h1)
        x, n2 = self.norm2.forward_with_residual(x, self.dropout(m))  # residual add fused with the norm
        return _ffn_residual(self, x, n2), new_state


class _TitansLM(nn.Module):
    """Embedding -> blocks -> RMSNorm -> tied head."""

    block_cls: type[nn.Module]
    model_type: str

    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.embed = nn.Embedding(config.vocab_size, config.dim)
        self.blocks = nn.ModuleList(self.block_cls(config) for _ in range(config.num_layers))
        self.norm = _norm(config)
        self.head = nn.Linear(config.dim, config.vocab_size, bias=False)
        self.head.weight = self.embed.weight
        nn.init.normal_(self.embed.weight, std=config.init_std)
        # derived weights (concatenations) shared by the segments of one forward
        self._wcache: dict = {}
        for mod in self.modules():
            if hasattr(type(mod), "_wcache") and mod is not self:
                mod._wcache = self._wcache

    def _run_blocks(self, x, states):
        new_states = []
        for block, st in zip(self.blocks, states, strict=True):
            x, ns = block(x, state=st)
            new_states.append(ns)
        return x, new_states

    def hidden_states(self, input_ids: torch.Tensor, states=None):
        """Final-norm hidden states [B, T, D] and new memory states (no head GEMM)."""
        if states is None:
            states = [None] * len(self.blocks)
        self._wcache.clear()
        self._wcache["active"] = True  # only while this forward runs
        try:
            x, new_states = self._run_blocks(self.embed(input_ids), states)
        finally:
            self._wcache.clear()  # weights change between forwards
        return self.norm(x), new_states

    def forward(self, input_ids: torch.Tensor, states: list[MemoryState] | None = None):
        h, new_states = self.hidden_states(input_ids, states)
        return linear(h, self.head.weight, use_kernels=self.config.use_kernels), new_states


class _StreamHandoff(torch.autograd.Function):
    """Identity at a stream boundary of the wavefront: ``x`` made on stream
    ``src`` is read on ``dst`` (the stream current in the forward).  Both
    directions tell the caching allocator about the other stream, so neither
    the activation nor its gradient (made on ``dst`` in the backward, read by
    the producer's backward on ``src``) is reused while the reader may still
    run."""

    @staticmethod
    def forward(ctx, x, src, dst):
        x.record_stream(dst)
        ctx.src = src
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g.record_stream(ctx.src)
        return g, None, None


class TitansMAC(_TitansLM):
    block_cls = MACBlock
    model_type = "mac"

    # Streams of the (layer, segment) wavefront; 0 = the sequential loop.
    wavefront_streams = 0

    def hidden_states(self, input_ids: torch.Tensor, states=None):
        if states is None:
            states = [None] * len(self.blocks)
        x = self.embed(input_ids)
        cs = self.config.chunk_size
        outs = []
        self._wcache.clear()
        self._wcache["active"] = True  # only while this forward runs
        try:
            if self.wavefront_streams > 1 and x.is_cuda and x.shape[1] > cs and len(self.blocks) > 1:
                outs, states = self._wavefront(x, list(states))
            else:
                for s in range(0, x.shape[1], cs):
                    chunk, states = self._run_blocks(x[:, s:s + cs], states)
                    outs.append(chunk)
        finally:
            self._wcache.clear()  # weights change between forwards
        return self.norm(torch.cat(outs, dim=1)), states

    def _wavefront(self, x: torch.Tensor, states: list):
        """The chunk loop as a (layer, segment) wavefront on CUDA streams.

        Block i on segment c needs block i-1's output on segment c and block
        i's memory state after segment c-1, nothing else (the reference's loop,
        `src/titans/models.py:301-314`, runs the same pairs one at a time).
        Block i runs on stream ``i mod n`` in segment order, and an event
        orders it after block i-1 on the same segment, so the pairs of one
        anti-diagonal (i + c constant) can run at the same time.  Every block
        still sees its segments in order, which also keeps the in-place writes
        of the memory state into its parameters in the sequential order.  The
        backward runs each op on its forward op's stream; :meth:`join_streams`
        makes the current stream wait for all of them.
        """
        main = torch.cuda.current_stream(x.device)
        streams = self._streams(x.device)
        for st in streams:
            st.wait_stream(main)
        cs = self.config.chunk_size
        cur = [x[:, s:s + cs] for s in range(0, x.shape[1], cs)]
        ready = [None] * len(cur)
        made_on = [main] * len(cur)
        L = len(self.blocks)
        for d in range(len(cur) + L - 1):
            for i in range(max(0, d - len(cur) + 1), min(d, L - 1) + 1):
                c = d - i
                st = streams[i % len(streams)]
                with torch.cuda.stream(st):
                    if ready[c] is not None:
                        st.wait_event(ready[c])
                    inp = cur[c] if made_on[c] is st else _StreamHandoff.apply(cur[c], made_on[c], st)
                    out, states[i] = self.blocks[i](inp, state=states[i])
                    ev = torch.cuda.Event()
                    ev.record(st)
                cur[c], ready[c], made_on[c] = out, ev, st
        self.join_streams()
        cur = [_StreamHandoff.apply(t, src, main) for t, src in zip(cur, made_on, strict=True)]
        for st_ in states:
            for t in st_.weights + st_.momentum:
                t.record_stream(main)
        return cur, states

    def _streams(self, device) -> list:
        n = int(self.wavefront_streams)
        have = getattr(self, "_wf_streams", None)
        if not have or len(have) != n or have[0].device != device:
            self._wf_streams = [torch.cuda.Stream(device) for _ in range(n)]
        return self._wf_streams

    def join_streams(self) -> None:
        """Make the current stream wait for the wavefront streams (after a
        forward, and after the backward before anything reads gradients)."""
        streams = getattr(self, "_wf_streams", None)
        if not streams:
            return
        main = torch.cuda.current_stream(streams[0].device)
        for st in streams:
            main.wait_stream(st)


class TitansMAG(_TitansLM):
    block_cls = MAGBlock
    model_type = "mag"


class TitansMAL(_TitansLM):
    block_cls = MALBlock
    model_type = "mal"


class TitansLMM(_TitansLM):
    block_cls = LMMBlock
    model_type = "lmm"


MODEL_CLASSES = {"mac": TitansMAC, "mag": TitansMAG, "mal": TitansMAL, "lmm": TitansLMM}


def create_model(model_type: str, config: TitansConfig) -> _TitansLM:
    try:
        return MODEL_CLASSES[model_type.lower()](config)
    except KeyError:
        raise ValueError(f"Unknown model type: {model_type}") from None
