"""Memory-update microbenchmark: the chunked neural-memory scan with per-token gates.

    python -m titans_pytorch_b200.cli.memory_bench                 # fused sm_100a kernel
    python -m titans_pytorch_b200.cli.memory_bench --impl torch    # same math in PyTorch ops

Workload (defaults): B=8 samples x H=16 heads = 128 independent memories, each
a 2-layer MLP 64 -> 256 -> 64 (fp32 weights and momentum, N(0, 0.02) init,
zero momentum); T=32768 tokens in chunks of 64; k, v, q ~ N(0, 1) then
l2-normalised over the 64 channels; per-token gates theta, eta, alpha =
sigmoid(N(0, 1)).  One step = the whole scan: retrieval of every query with
the memory at its chunk's start, and the update of every chunk (forward on
the keys, loss gradient, both weight-gradient GEMMs with the folded
coefficients, momentum and decay).

``--impl torch`` is the baseline: the same chunked math written with PyTorch
ops (batched matmuls over the 128 memories, looped over the 512 chunks), the
way the reference's per-call update (`memory.py:287-351, 464-498`) would be
vectorised over (batch, head) on the same GPU.  Timing: CUDA events around each
step after ``--warmup`` steps; the state buffers (128 x 4 x 64 KB) are rewritten
every chunk, and the inputs (3 x 512 MB bf16 at the defaults) exceed the L2.
One JSON line: ms per step, memory-token updates per second, TFLOP/s
(2 * 5 * 128 * 256 * 64 per chunk and memory: the five 128x256x64-equivalent
products) and the fraction of the given bf16 peak.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch


def make_inputs(B: int, H: int, T: int, d: int, hidden: int, device, seed: int = 0):
    g = torch.Generator(device=device).manual_seed(seed)
    N = B * H

    def unit(*shape):
        x = torch.randn(*shape, device=device, generator=g)
        return torch.nn.functional.normalize(x, dim=-1).to(torch.bfloat16)

    k, v, q = unit(N, T, d), unit(N, T, d), unit(N, T, d)
    theta, eta, alpha = (torch.sigmoid(torch.randn(N, T, device=device, generator=g)) for _ in range(3))
    W = [torch.randn(N, hidden, d, device=device, generator=g) * 0.02,
         torch.randn(N, d, hidden, device=device, generator=g) * 0.02]
    S = [torch.zeros_like(w) for w in W]
    return W, S, k, v, q, theta, eta, alpha


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Chunked memory-scan microbenchmark")
    add = p.add_argument
    add("--impl", choices=["ours", "torch"], default="ours")
    add("--batch", type=int, default=8)
    add("--heads", type=int, default=16)
    add("--seq", type=int, default=32768)
    add("--dim", type=int, default=64)
    add("--hidden", type=int, default=256)
    add("--chunk", type=int, default=64)
    add("--mode", choices=["paper", "ref"], default="paper",
        help="paper: the chunked per-head scan above; ref: one reference-semantics update of a "
             "block's memory (memory_step: MLP forward on the keys, scaled error, back-propagation, "
             "gated update in the weight-gradient epilogues) at a training workload's shape")
    add("--shape", choices=["mag170m", "mal760m"], default="mag170m", help="--mode ref: workload shape")
    add("--warmup", type=int, default=1)
    add("--steps", type=int, default=3)
    add("--peak-tflops", type=float, default=None, help="bf16 GEMM burst peak (default: the measured one)")
    a = p.parse_args(argv)
    from ..utils.perf import measured_peaks

    peaks = measured_peaks()
    if a.peak_tflops is None:
        a.peak_tflops = peaks["bf16_tflops"]
    if getattr(a, "peak_gbs", 0) is None:
        a.peak_gbs = peaks["hbm_gbs"]
    if a.mode == "ref":
        ref_update(a)
        return
    from ..ops.memory_paper import memory_scan

    dev = torch.device("cuda")
    W, S, k, v, q, theta, eta, alpha = make_inputs(a.batch, a.heads, a.seq, a.dim, a.hidden, dev)
    use = a.impl == "ours"

    def step():
        return memory_scan(W, S, k, v, q, theta, eta, alpha, a.chunk, "silu", use_kernels=use)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        y, W1, S1 = step()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    ms = statistics.median(times)
    N = a.batch * a.heads
    chunks = (a.seq + a.chunk - 1) // a.chunk
    flops = 2.0 * 5 * 128 * a.hidden * a.dim * chunks * N
    tf = flops / ms / 1e9
    rec = {"bench": "memory_scan", "impl": a.impl, "ms": round(ms, 3),
           "memory_tokens_per_s": N * a.seq / ms * 1e3, "tflops": round(tf, 1),
           "frac_of_measured_peak": round(tf / a.peak_tflops, 4),
           "config": {"B": a.batch, "H": a.heads, "T": a.seq, "d": a.dim, "hidden": a.hidden, "chunk": a.chunk},
           "y_finite": bool(torch.isfinite(y.float()).all()), "state_norm": float(W1[0].float().norm())}
    if use:
        from ..ops._ext import ext

        rec["kernel_error_status"] = int(ext().kernel_error_status(0, True))
    print(json.dumps(rec))


REF_SHAPES = {  # tokens per update (micro-batch x sequence), dim, memory hidden width, memory depth
    "mag170m": dict(B=8, T=4096, D=768, hidden=3072, L=2),
    "mal760m": dict(B=1, T=16384, D=1536, hidden=6144, L=3),
}


def ref_update(a) -> None:
    """Time ``memory_step`` (reference semantics) at a training workload's shape.

    FLOPs = 2 N (3 S - d0 d1) with N tokens and S = sum of the layers' d_i d_{i+1}:
    the forward GEMMs, every weight-gradient GEMM, and the input-gradient GEMMs
    of all layers but the first; the bound is compute (all GEMMs are large),
    so the roofline time is FLOPs / the measured bf16 peak."""
    from ..ops._ext import ext
    from ..ops.memory import memory_step

    sh = REF_SHAPES[a.shape]
    B, T, D, Hd, L = sh["B"], sh["T"], sh["D"], sh["hidden"], sh["L"]
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    k = torch.nn.functional.normalize(torch.randn(B, T, D, device=dev, generator=g), dim=-1).to(bf)
    v = torch.randn(B, T, D, device=dev, generator=g).to(bf)
    x = torch.randn(B, T, D, device=dev, generator=g).to(bf)
    dims = [D] + [Hd] * (L - 1) + [D]
    ws = [(0.02 * torch.randn(dims[i + 1], dims[i], device=dev, generator=g)).to(bf) for i in range(L)]
    ms = [torch.zeros_like(w) for w in ws]
    gw = [(0.02 * torch.randn(D, D, device=dev, generator=g)).to(bf) for _ in range(3)]
    gb = [torch.zeros(D, device=dev, dtype=bf) for _ in range(3)]

    def step():
        return memory_step(k, v, x, ws, ms, gw, gb, 0.1, 0.9, "silu")

    for _ in range(max(1, a.warmup)):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        nw, nm = step()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    ms_ = statistics.median(times)
    N = B * T
    S = sum(dims[i] * dims[i + 1] for i in range(L))
    flops = 2.0 * N * (3 * S - dims[0] * dims[1])
    tf = flops / ms_ / 1e9
    print(json.dumps({"bench": "memory_update_ref", "shape": a.shape, "ms": round(ms_, 4),
                      "gflop": round(flops / 1e9, 1), "tflops": round(tf, 1),
                      "frac_of_measured_peak": round(tf / a.peak_tflops, 3),
                      "roofline_ms": round(flops / a.peak_tflops / 1e9, 4),
                      "config": {"B": B, "T": T, "D": D, "hidden": Hd, "L_M": L},
                      "state_finite": bool(all(torch.isfinite(t.float()).all() for t in nw + nm)),
                      "kernel_error_status": int(ext().kernel_error_status(0, True))}))


if __name__ == "__main__":
    main()
