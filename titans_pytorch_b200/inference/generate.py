"""Autoregressive generation for Titans models.

Reference behaviour (`scripts/inference.py:321-423`,
`src/titans/optimized_inference.py:143-345`): every new token re-runs the model
on the last ``chunk_size`` tokens with the memory states carried from the
previous call, then samples with temperature / repetition penalty / top-k /
top-p.  That recurrence defines the model's outputs, so it is kept; what
changes here is that each step is one batched forward through the sm_100a
kernels, the sampling filters are vectorised (no per-token Python loops over
the vocabulary), and the EOS test touches the host once per step only when an
EOS id is given.

``repetition_penalty`` follows the reference exactly: the logits of tokens
already generated are divided by the penalty (whatever their sign).
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Iterator

import torch
import torch.nn.functional as F


# ----------------------------------------------------------------- sampling
def apply_repetition_penalty(logits: torch.Tensor, generated: torch.Tensor, penalty: float) -> torch.Tensor:
    if penalty == 1.0:
        return logits
    seen = torch.zeros_like(logits, dtype=torch.bool).scatter_(1, generated, True)
    return torch.where(seen, logits / penalty, logits)


def top_k_filter(logits: torch.Tensor, k: int) -> torch.Tensor:
    if k <= 0 or k >= logits.shape[-1]:
        return logits
    kth = torch.topk(logits, k)[0][..., -1, None]
    return logits.masked_fill(logits < kth, float("-inf"))


def top_p_filter(logits: torch.Tensor, p: float) -> torch.Tensor:
    if p >= 1.0:
        return logits
    sorted_logits, idx = torch.sort(logits, descending=True)
    cum = torch.cumsum(F.softmax(sorted_logits, dim=-1), dim=-1)
    remove = cum > p
    remove[..., 1:] = remove[..., :-1].clone()
    remove[..., 0] = False
    return logits.masked_fill(remove.scatter(1, idx, remove), float("-inf"))


def sample_next(logits: torch.Tensor, generated: torch.Tensor, temperature: float = 1.0, top_k: int = 50,
                top_p: float = 0.9, repetition_penalty: float = 1.0, greedy: bool = False,
                generator: torch.Generator | None = None) -> torch.Tensor:
    """Next token ids [B, 1] from last-position logits [B, V]."""
    logits = logits.float() / max(temperature, 1e-7)
    logits = apply_repetition_penalty(logits, generated, repetition_penalty)
    if greedy:
        return logits.argmax(dim=-1, keepdim=True)
    logits = top_p_filter(top_k_filter(logits, top_k), top_p)
    return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1, generator=generator)


# --------------------------------------------------------------- generation
def _context(model, generated: torch.Tensor, context_size: int | None) -> torch.Tensor:
    n = context_size or model.config.chunk_size
    return generated[:, -min(generated.shape[1], n):]


@torch.no_grad()
def generate(model, input_ids: torch.Tensor, max_new_tokens: int = 100, temperature: float = 1.0,
             top_k: int = 50, top_p: float = 0.9, repetition_penalty: float = 1.0,
             eos_token_id: int | None = None, states=None, stream: bool = False, greedy: bool = False,
             context_size: int | None = None, generator: torch.Generator | None = None):
    """Generate tokens; returns ``(ids, states)`` or, with ``stream=True``, an iterator of them."""
    def steps() -> Iterator:
        nonlocal states
        generated = input_ids.clone()
        for _ in range(max_new_tokens):
            logits, states = model(_context(model, generated, context_size), states=states)
            nxt = sample_next(logits[:, -1, :], generated, temperature, top_k, top_p, repetition_penalty,
                              greedy, generator)
            generated = torch.cat([generated, nxt.to(generated.dtype)], dim=1)
            done = eos_token_id is not None and bool((nxt == eos_token_id).all())
            if stream:
                yield generated, states
            if done:
                break
        if not stream:
            yield generated, states

    it = steps()
    return it if stream else next(it)


@torch.no_grad()
def prefill(model, input_ids: torch.Tensor, states=None, chunk: int | None = None):
    """Run a long prompt through the model chunk by chunk with carried states.

    Returns ``(last_logits [B, V], states)``.  For MAC the model chunks by
    ``chunk_size`` internally; for the other variants each chunk is one
    memory update (the reference's streaming evaluation,
    `scripts/eval_perplexity.py:263-339`).
    """
    chunk = chunk or model.config.chunk_size
    last = None
    for s in range(0, input_ids.shape[1], chunk):
        logits, states = model(input_ids[:, s:s + chunk], states=states)
        last = logits[:, -1, :]
    return last, states


class GraphedForward:
    """``model(x, states)`` for one fixed input shape, captured in a CUDA graph.

    The memory states are chained in place: each replay reads the states the
    previous replay left in ``self.states`` and overwrites them with the new
    ones, so prefilling a long prompt or decoding token by token is a series of
    replays with only an input copy in between.  ``states`` (from an eager call
    of the same model) seeds the chain; it is copied, not kept.
    """

    def __init__(self, model, batch: int, length: int, states, warmup: int = 2) -> None:
        dev = next(model.parameters()).device
        self.x = torch.zeros(batch, length, dtype=torch.long, device=dev)
        self.states = [s.clone() for s in states]
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(cur)
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(warmup):
                model(self.x, states=[s.clone() for s in self.states])
        cur.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            logits, new = model(self.x, states=self.states)
            for old, nxt in zip(self.states, new):
                for a, b in zip(old.weights + old.momentum, nxt.weights + nxt.momentum):
                    a.copy_(b)
        self.logits = logits

    def load_states(self, states) -> None:
        for old, nxt in zip(self.states, states):
            for a, b in zip(old.weights + old.momentum, nxt.weights + nxt.momentum):
                a.copy_(b)

    def __call__(self, x: torch.Tensor):
        """Returns ``(logits, states)``; both are overwritten by the next call."""
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.logits, self.states


class OptimizedGenerator:
    """Generation front-end (`src/titans/optimized_inference.py:143-345`)."""

    def __init__(self, model, device=None, dtype: torch.dtype | None = None) -> None:
        self.model = model
        if device is not None or dtype is not None:
            self.model = model.to(device=device, dtype=dtype)
        self.model.eval()

    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100, **kw):
        return generate(self.model, input_ids, max_new_tokens, **kw)

    def generate_streaming(self, input_ids: torch.Tensor, max_new_tokens: int = 100, **kw):
        """Yield one new token id tensor [B, 1] at a time."""
        for ids, _ in generate(self.model, input_ids, max_new_tokens, stream=True, **kw):
            yield ids[:, -1:]


# ------------------------------------------------------------- static cache
@dataclass
class KVCacheConfig:
    max_batch_size: int = 8
    max_seq_len: int = 4096
    num_layers: int = 12
    num_heads: int = 8
    head_dim: int = 64
    dtype: torch.dtype = torch.bfloat16


class StaticKVCache:
    """Preallocated per-layer K/V buffers with per-sequence lengths.

    Kept for API parity with the reference (`optimized_inference.py:46-135`),
    where the models never consume it either; the Titans models here recompute
    the attention context from the token window on every call.
    """

    def __init__(self, config: KVCacheConfig, device=None) -> None:
        c = config
        shape = (c.num_layers, c.max_batch_size, c.num_heads, c.max_seq_len, c.head_dim)
        self.config = c
        self.k = torch.zeros(shape, dtype=c.dtype, device=device)
        self.v = torch.zeros(shape, dtype=c.dtype, device=device)
        self.seq_lens = torch.zeros(c.max_batch_size, dtype=torch.long, device=device)

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor, batch_indices: torch.Tensor):
        """Append k/v [b, H, t, d] for the given sequences; returns the cached K/V."""
        t = k.shape[2]
        for j, bi in enumerate(batch_indices.tolist()):
            s = int(self.seq_lens[bi])
            if s + t > self.config.max_seq_len:
                raise ValueError("StaticKVCache overflow")
            self.k[layer, bi, :, s:s + t] = k[j]
            self.v[layer, bi, :, s:s + t] = v[j]
        n = int(self.seq_lens[batch_indices].max()) + t
        return self.k[layer, batch_indices, :, :n], self.v[layer, batch_indices, :, :n]

    def increment_seq_len(self, batch_indices: torch.Tensor, delta: int) -> None:
        self.seq_lens[batch_indices] += delta

    def reset(self, batch_indices: torch.Tensor | None = None) -> None:
        if batch_indices is None:
            self.seq_lens.zero_()
        else:
            self.seq_lens[batch_indices] = 0


# -------------------------------------------------------- continuous batching
class ContinuousBatcher:
    """Serve many requests with one batched forward per step.

    Like the reference (`optimized_inference.py:353-473`) each step re-runs the
    model on (up to) the last ``context`` tokens of every active request,
    left-padded to a common length, and memory states are not carried between
    steps.  Finished requests leave the batch and new ones join at any step.
    """

    def __init__(self, model, max_batch_size: int = 8, context: int = 512, pad_token_id: int = 0,
                 device=None) -> None:
        self.model = model
        self.max_batch_size = max_batch_size
        self.context = context
        self.pad = pad_token_id
        self.device = device or next(model.parameters()).device
        self.queue: list[dict] = []
        self.active: list[dict] = []
        self._next_id = 0

    def add_request(self, input_ids: torch.Tensor, max_new_tokens: int = 50, temperature: float = 1.0,
                    top_k: int = 50, top_p: float = 0.9, eos_token_id: int | None = None) -> int:
        rid = self._next_id
        self._next_id += 1
        self.queue.append(dict(id=rid, ids=input_ids.reshape(-1).to(self.device), left=max_new_tokens,
                               temperature=temperature, top_k=top_k, top_p=top_p, eos=eos_token_id))
        return rid

    @torch.no_grad()
    def step(self) -> list[dict]:
        """One decoding step for every active request; returns the requests that finished."""
        while self.queue and len(self.active) < self.max_batch_size:
            self.active.append(self.queue.pop(0))
        if not self.active:
            return []
        ctx = [r["ids"][-self.context:] for r in self.active]
        n = max(c.numel() for c in ctx)
        batch = torch.full((len(ctx), n), self.pad, dtype=torch.long, device=self.device)
        for i, c in enumerate(ctx):
            batch[i, n - c.numel():] = c
        logits, _ = self.model(batch)
        last = logits[:, -1, :]
        finished, keep = [], []
        for i, r in enumerate(self.active):
            nxt = sample_next(last[i:i + 1], r["ids"][None], r["temperature"], r["top_k"], r["top_p"])
            r["ids"] = torch.cat([r["ids"], nxt.reshape(-1)])
            r["left"] -= 1
            if r["left"] <= 0 or (r["eos"] is not None and int(nxt) == r["eos"]):
                finished.append({"id": r["id"], "ids": r["ids"]})
            else:
                keep.append(r)
        self.active = keep
        return finished

    def run(self) -> list[dict]:
        out = []
        while self.queue or self.active:
            out += self.step()
        return out


# ------------------------------------------------------------- quantization
@torch.no_grad()
def quantize_model_dynamic(model, bits: int = 8):
    """Weight-only symmetric per-output-channel quantization (the reference's
    ``quantize_model_dynamic``, `optimized_inference.py:481-536`).

    ``bits=8``: real int8 weights (:func:`~titans_pytorch_b200.ops.quant.quantize_model_int8`):
    half the bf16 bytes in memory, dequantised inside the int8 GEMM.  Other
    widths round the weights to the ``bits``-bit grid and store them back in
    their dtype (the numerics of the quantized weights, no memory saving).
    """
    if bits == 8:
        from ..ops.quant import quantize_model_int8

        return quantize_model_int8(model)
    qmax = 2 ** (bits - 1) - 1
    for m in model.modules():
        if isinstance(m, torch.nn.Linear):
            w = m.weight.data.float()
            scale = w.abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / qmax
            m.weight.data.copy_((torch.round(w / scale).clamp_(-qmax, qmax) * scale).to(m.weight.dtype))
    return model


quantize_model_static = quantize_model_dynamic


def benchmark_generation(model, batch_size: int = 1, prompt_len: int = 128, gen_len: int = 64,
                         vocab_size: int | None = None, warmup: int = 2) -> dict[str, float]:
    """Prefill and decode throughput (tokens/s) with device timing."""
    dev = next(model.parameters()).device
    V = vocab_size or model.config.vocab_size
    ids = torch.randint(0, V, (batch_size, prompt_len), device=dev)
    for _ in range(warmup):
        generate(model, ids, 2, greedy=True)
    sync = torch.cuda.synchronize if dev.type == "cuda" else (lambda: None)
    sync()
    t0 = time.perf_counter()
    _, st = prefill(model, ids)
    sync()
    t1 = time.perf_counter()
    generate(model, ids, gen_len, greedy=True, states=st)
    sync()
    t2 = time.perf_counter()
    return {"prefill_tokens_per_s": batch_size * prompt_len / (t1 - t0),
            "decode_tokens_per_s": batch_size * gen_len / (t2 - t1)}
