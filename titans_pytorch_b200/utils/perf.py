"""Runtime utilities: device timers, NVTX ranges, memory stats, model benchmarks,
activation checkpointing and CUDA-graph capture.

Counterparts of the reference's helpers (`src/titans/cuda_optimizations.py:378-759`,
`src/titans/optimized_training.py:428-603`) with B200-specific choices:

* ``compile_model`` does not run torch.compile; it returns a
  :class:`CUDAGraphRunner` that captures the model's forward for fixed input
  shapes and replays it (launch overhead is the cost torch.compile's
  ``reduce-overhead`` mode targets).
* ``configure_memory_pool`` does **not** claim a fraction of the GPU (the
  reference sets 0.95, which starves other processes on a shared device); it
  only sets allocator options that take effect before the first allocation.
* timing is CUDA events on the launching stream, never wall clock.
"""

from __future__ import annotations

import contextlib
import os
import subprocess
import time

import torch

try:  # NVTX ranges for nsys/ncu timelines
    import torch.cuda.nvtx as _nvtx
except Exception:  # pragma: no cover
    _nvtx = None


@contextlib.contextmanager
def nvtx_range(name: str):
    if _nvtx is not None and torch.cuda.is_available():
        _nvtx.range_push(name)
        try:
            yield
        finally:
            _nvtx.range_pop()
    else:
        yield


class CudaTimer:
    """Accumulates device time of regions with CUDA events (read with ``.ms``)."""

    def __init__(self) -> None:
        self.events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    @contextlib.contextmanager
    def region(self):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        self.events.append((s, e))

    @property
    def ms(self) -> float:
        torch.cuda.synchronize()
        return sum(s.elapsed_time(e) for s, e in self.events)


@contextlib.contextmanager
def profile_cuda(name: str = "profile", enabled: bool = True, sink=print):
    """Print the device time of the enclosed region (CUDA events)."""
    if not enabled or not torch.cuda.is_available():
        yield
        return
    t = CudaTimer()
    with nvtx_range(name), t.region():
        yield
    sink(f"{name}: {t.ms:.3f} ms")


def get_gpu_memory_stats(device=None) -> dict[str, float]:
    if not torch.cuda.is_available():
        return {}
    gb = 1024 ** 3
    return {"allocated_gb": torch.cuda.memory_allocated(device) / gb,
            "reserved_gb": torch.cuda.memory_reserved(device) / gb,
            "max_allocated_gb": torch.cuda.max_memory_allocated(device) / gb}


def print_gpu_utilization() -> str:
    """nvidia-smi utilisation / memory / clocks (read-only query)."""
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=index,utilization.gpu,memory.used,memory.total,"
                              "clocks.sm,clocks.max.sm,power.draw", "--format=csv"],
                             capture_output=True, text=True, timeout=10).stdout
    except (OSError, subprocess.SubprocessError) as e:
        out = f"nvidia-smi unavailable: {e}"
    print(out)
    return out


def configure_memory_pool(expandable_segments: bool = True) -> None:
    """Allocator options only (no per-process memory fraction on shared GPUs)."""
    if expandable_segments and "PYTORCH_CUDA_ALLOC_CONF" not in os.environ:
        os.environ["PYTORCH_CUDA_ALLOC_CONF"] = "expandable_segments:True"


def empty_cache_if_needed(threshold: float = 0.9) -> None:
    if torch.cuda.is_available():
        free, total = torch.cuda.mem_get_info()
        if 1 - free / total > threshold:
            torch.cuda.empty_cache()


def enable_wavefront(model: torch.nn.Module, streams: int = 2) -> torch.nn.Module:
    """Run a MAC model's (layer, segment) loop as a wavefront on ``streams``
    CUDA streams (``streams <= 1``: the sequential loop).  The result is the
    sequential loop's; the pairs (i, c) with equal i + c may run concurrently,
    which fills the GPU better when each segment's kernels are small."""
    if getattr(model, "model_type", None) != "mac":
        raise ValueError("the wavefront schedule is for MAC models (segments x layers)")
    model.wavefront_streams = int(streams)
    return model


def enable_gradient_checkpointing(model: torch.nn.Module) -> torch.nn.Module:
    """Recompute each block's forward in the backward (non-reentrant checkpoint).

    The memory update has no gradient (its output, the next state, is
    detached), so for blocks whose memory reads the block input (MAG, MAL,
    LMM; reference semantics) it runs once, under ``no_grad`` before the
    checkpointed region, and the region (recomputed in the backward) skips it.
    Other blocks recompute their whole forward; the update is a pure function
    of the block input, so the recomputation reproduces it exactly.
    """
    from torch.utils.checkpoint import checkpoint

    for block in getattr(model, "blocks", []):
        if getattr(block, "_titans_ckpt", False):
            continue
        fwd = block.forward
        split = hasattr(block, "memory_input") and getattr(block.memory, "paper", False) is False

        if split:
            def wrapped(x, state=None, _fwd=fwd, _blk=block):
                mem = _blk.memory
                if state is None:
                    state = mem.init_state(x.shape[0], x.device)
                with torch.no_grad():
                    n = _blk.memory_input(x)
                    h = 0
                    if getattr(_blk, "cp", None) is not None:  # context parallel: the convolutions' halo
                        from ..models.titans import _conv_halo, _halo
                        n, h, _ = _halo(_blk, n, _conv_halo(_blk.config))
                    new_state = mem._update(n, state, h)
                out = checkpoint(lambda xx, st: _fwd(xx, st, update_memory=False)[0], x, state, use_reentrant=False)
                return out, new_state
        else:
            def wrapped(x, state=None, _fwd=fwd):
                return checkpoint(_fwd, x, state, use_reentrant=False)

        block.forward = wrapped
        block._titans_ckpt = True
    return model


class CUDAGraphRunner:
    """Capture ``fn(*static_inputs)`` once and replay it; inputs are copied into static buffers."""

    def __init__(self, fn, example_inputs: tuple[torch.Tensor, ...], warmup: int = 2) -> None:
        self.fn = fn
        self.static_in = tuple(x.clone() for x in example_inputs)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn(*self.static_in)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_out = fn(*self.static_in)

    def __call__(self, *inputs: torch.Tensor):
        for dst, src in zip(self.static_in, inputs):
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.static_out


def compile_model(model: torch.nn.Module, example_input_ids: torch.Tensor | None = None, **_ignored):
    """Inference forward captured as a CUDA graph for ``example_input_ids``'s shape
    (returns the model unchanged without an example or without CUDA)."""
    if example_input_ids is None or not torch.cuda.is_available():
        return model
    model.eval()

    @torch.no_grad()
    def fwd(ids):
        return model(ids)[0]

    return CUDAGraphRunner(fwd, (example_input_ids,))


def compile_function(fn, *_args, **_kw):
    return fn


@torch.no_grad()
def benchmark_model(model: torch.nn.Module, batch_size: int = 4, seq_len: int = 256, warmup: int = 3,
                    iters: int = 10, vocab_size: int | None = None) -> dict[str, float]:
    """Forward latency (ms) and tokens/s, device-timed."""
    dev = next(model.parameters()).device
    ids = torch.randint(0, vocab_size or model.config.vocab_size, (batch_size, seq_len), device=dev)
    model.eval()
    for _ in range(warmup):
        model(ids)
    if dev.type == "cuda":
        t = CudaTimer()
        with t.region():
            for _ in range(iters):
                model(ids)
        ms = t.ms / iters
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            model(ids)
        ms = (time.perf_counter() - t0) * 1000 / iters
    return {"latency_ms": ms, "tokens_per_s": batch_size * seq_len / (ms / 1000)}


def get_optimal_batch_size(model: torch.nn.Module, seq_len: int, max_batch: int = 256,
                           memory_fraction: float = 0.8) -> int:
    """Largest power-of-two batch whose training step fits in ``memory_fraction`` of free memory."""
    if not torch.cuda.is_available():
        return 1
    dev = next(model.parameters()).device
    best, b = 1, 1
    free0 = torch.cuda.mem_get_info(dev)[0]
    while b <= max_batch:
        try:
            torch.cuda.reset_peak_memory_stats(dev)
            base = torch.cuda.memory_allocated(dev)
            ids = torch.randint(0, model.config.vocab_size, (b, seq_len), device=dev)
            logits, _ = model(ids)
            logits.float().mean().backward()
            model.zero_grad(set_to_none=True)
            if torch.cuda.max_memory_allocated(dev) - base > memory_fraction * free0:
                break
            best = b
            b *= 2
        except torch.cuda.OutOfMemoryError:
            break
        finally:
            torch.cuda.empty_cache()
    return best


def is_triton_available() -> bool:
    """The framework's kernels are native CUDA; Triton is never used."""
    return False


def is_flash_attention_available() -> bool:
    """True: attention runs on the framework's own sm_100a flash kernels."""
    from ..ops._ext import available

    return available()


def is_torch_sdpa_available() -> bool:
    return hasattr(torch.nn.functional, "scaled_dot_product_attention")


# ---------------------------------------------------------------- fused helpers and streams
# (`src/titans/cuda_optimizations.py:37-148, 547-644` surface)
from ..ops.norm import fused_add_rms_norm  # noqa: E402  (kernel-backed residual add + RMSNorm)


def fused_silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up: one elementwise kernel on CUDA (the reference's
    `cuda_optimizations.py:118-125` is two PyTorch ops).  Tensors that need a
    gradient, or that the kernel cannot take, use the PyTorch definition."""
    from ..ops._ext import want_kernels

    if (want_kernels(gate) and gate.shape == up.shape and gate.dtype == up.dtype
            and gate.dtype in (torch.bfloat16, torch.float16, torch.float32)
            and gate.shape[-1] % (16 // gate.element_size()) == 0
            and not (torch.is_grad_enabled() and (gate.requires_grad or up.requires_grad))):
        from ..ops._ext import ext

        return ext().silu_mul(gate, up)
    return torch.nn.functional.silu(gate) * up


def fused_linear_silu_linear(x: torch.Tensor, gate_weight: torch.Tensor, up_weight: torch.Tensor,
                             down_weight: torch.Tensor) -> torch.Tensor:
    """down(silu(x gate^T) * (x up^T)): the SwiGLU FFN (one stacked gate|up GEMM and
    the SiLU-product kernel on CUDA)."""
    from ..ops.ffn import swiglu_ffn

    return swiglu_ffn(x, gate_weight, up_weight, down_weight)


class CUDAStreamManager:
    """A small pool of CUDA streams: ``with mgr.stream(i): ...`` runs work on
    stream i; ``synchronize()`` joins every stream into the current one."""

    def __init__(self, num_streams: int = 3) -> None:
        self.enabled = torch.cuda.is_available()
        self.streams = [torch.cuda.Stream() for _ in range(num_streams)] if self.enabled else []

    @contextlib.contextmanager
    def stream(self, stream_id: int = 0):
        if not self.enabled:
            yield None
            return
        s = self.streams[stream_id % len(self.streams)]
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            yield s

    def synchronize(self) -> None:
        if self.enabled:
            cur = torch.cuda.current_stream()
            for s in self.streams:
                cur.wait_stream(s)


@torch.no_grad()
def optimized_generate_step(model, input_ids: torch.Tensor, states=None, context: int | None = None):
    """One decoding step: logits of the next token for the last ``context``
    tokens (default the model's chunk size) with the memory states carried.
    Returns ``(next_logits [B, V], new_states)``."""
    n = context or model.config.chunk_size
    logits, states = model(input_ids[:, -min(n, input_ids.shape[1]):], states=states)
    return logits[:, -1], states


@torch.no_grad()
def speculative_decode(model, draft_model, input_ids: torch.Tensor, num_speculative_tokens: int = 4,
                       max_new_tokens: int = 32, context: int | None = None) -> torch.Tensor:
    """Greedy speculative decoding over a sliding context window.

    The draft model proposes ``num_speculative_tokens`` tokens greedily; the
    target scores the window plus all proposals in ONE forward and keeps the
    longest prefix it agrees with, plus its own next token.  Neither model
    carries memory states.  When a model's output at a position depends only on
    its last ``context`` tokens, the result equals plain greedy decoding with that
    window. That holds for MAG / MAL / LMM with an attention window no larger than
    ``context``: without carried states the memory is read at its initial weights
    per position. It does not hold for MAC, whose segment memory tokens depend on
    the whole segment.
    """
    n = context or model.config.chunk_size
    out = input_ids
    while out.shape[1] - input_ids.shape[1] < max_new_tokens:
        draft = out
        for _ in range(num_speculative_tokens):
            lg, _ = draft_model(draft[:, -n:])
            draft = torch.cat([draft, lg[:, -1:].argmax(-1)], 1)
        k = draft.shape[1] - out.shape[1]
        span = draft[:, -(n + k):]
        lg, _ = model(span)
        choice = lg[:, -(k + 1):].argmax(-1)          # target's token after each proposal prefix
        proposed = draft[:, out.shape[1]:]
        agree = (choice[:, :k] == proposed).all(0)    # accept a position only if every row agrees
        m = int(agree.int().cumprod(0).sum())
        out = torch.cat([out, proposed[:, :m], choice[:, m:m + 1]], 1)
    return out[:, :input_ids.shape[1] + max_new_tokens]


def measured_peaks() -> dict:
    """Roofline denominators measured on the target B200s: ``MEASURED_PEAKS.json``
    at the repository root (``hbm_gbs`` copy rate, ``bf16_tflops`` cuBLAS burst,
    ``bf16_tflops_sustained``), else the earlier measurement on the same parts
    (6650 GB/s, 1590 / 1400 TFLOP/s).  ``source`` says which."""
    import json
    import os

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        out.update({k: float(d[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained") if k in d})
        out["source"] = "measured"
    except (OSError, ValueError):
        pass
    return out
