"""Per-kernel timings of the sm_100a extension on the flagship training shapes.

    python -m titans_pytorch_b200.cli.kernel_bench --op attn_bwd_tc --batch 2
    python -m titans_pytorch_b200.cli.kernel_bench --op all

Each op is timed with CUDA events on the launching stream after ``--warmup``
untimed launches; an L2 flush (a write of a buffer larger than the 126 MB L2)
runs between timed launches and is not inside the events.  One JSON line per
op: median milliseconds, achieved TFLOP/s (contractions) or GB/s (memory-bound
ops, algorithmic bytes), and the fraction of the given peaks.  The peak
defaults are the measured bf16 cuBLAS GEMM burst and device copy rate
(``MEASURED_PEAKS.json`` at the repository root).

Shapes default to the training benchmark's (dim 768, 12 heads of 64, sequence
4096, window 512, 4 persistent tokens); ``--batch`` is per launch.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

OPS = ("attn_fwd_tc", "attn_fwd_mma", "attn_bwd_tc", "attn_bwd_mma", "conv_fwd", "conv_bwd", "rms_fwd",
       "rms_bwd", "swiglu_fwd", "swiglu_bwd", "ce_fwd", "gemm_tc", "gemm_cublas", "gemm_gather")


def visible_pairs(T: int, W: int, P: int) -> int:
    """(query, key) pairs a sliding window of W over T tokens plus P prefix keys scores."""
    full = max(0, T - W)
    ramp = min(T, W)
    return ramp * (ramp + 1) // 2 + full * W + T * P


def time_op(fn, warmup: int, iters: int, flush: torch.Tensor | None) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.fill_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def build(op: str, a) -> tuple:
    """Returns (callable, flops, bytes) for one op on the configured shape."""
    from ..ops import _ext

    E = _ext.ext()
    dev, bf = torch.device("cuda"), torch.bfloat16
    B, H, T, P, W, d = a.batch, a.heads, a.seq, a.persistent, a.window, a.head_dim
    D = H * d
    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*shape, dtype=bf):
        return torch.randn(*shape, device=dev, dtype=dtype, generator=g)

    if op.startswith("attn"):
        Q, K, V = rn(B, H, T, d), rn(B, H, P + T, d), rn(B, H, P + T, d)
        scale = d ** -0.5
        fwd = E.attn_fwd_tc if op.endswith("_tc") else E.attn_fwd_packed
        pairs = B * H * visible_pairs(T, W, P)
        if "fwd" in op:
            return (lambda: fwd(Q, K, V, W, scale)), 4.0 * pairs * d, 0
        O, lse = E.attn_fwd_tc(Q, K, V, W, scale)
        dO = rn(*O.shape)
        bwd = E.attn_bwd_tc if op.endswith("_tc") else E.attn_bwd_packed
        return (lambda: bwd(dO, Q, K, V, O, lse, W, scale)), 10.0 * pairs * d, 0
    rows = B * T
    if op.startswith("conv"):
        x = rn(B, T, D)
        w, b = rn(4, D, dtype=torch.float32), rn(D, dtype=torch.float32)
        if op == "conv_fwd":
            return (lambda: E.conv_silu_norm_fwd(x, w, b, True)), 0, 2 * x.numel() * 2
        dy = rn(B, T, D)
        return (lambda: E.conv_silu_norm_bwd(dy, x, w, b, True, True)), 0, 3 * x.numel() * 2
    if op.startswith("rms"):
        x, w = rn(rows, D), torch.ones(D, device=dev, dtype=bf)
        if op == "rms_fwd":
            return (lambda: E.rms_norm_fwd(x, w, 1e-6)), 0, 2 * x.numel() * 2
        y, rstd = E.rms_norm_fwd(x, w, 1e-6)
        dy = rn(rows, D)
        return (lambda: E.rms_norm_bwd(dy, x, w, rstd, True)), 0, 3 * x.numel() * 2
    if op.startswith("swiglu"):
        F = int(D * a.ffn_mult)
        gu = rn(rows, 2 * F)
        if op == "swiglu_fwd":
            return (lambda: E.swiglu_fwd(gu)), 0, (gu.numel() + rows * F) * 2
        dh = rn(rows, F)
        return (lambda: E.swiglu_bwd(dh, gu)), 0, (2 * gu.numel() + dh.numel()) * 2
    if op == "ce_fwd":
        logits = rn(rows, a.vocab)
        labels = torch.randint(0, a.vocab, (rows,), device=dev, generator=g)
        return (lambda: E.cross_entropy_fwd(logits, labels, -100)), 0, logits.numel() * 2
    if op.startswith("gemm"):
        # the first projection of a layer: [B*T, D] x [3D, D]^T (q|k|v)
        M, N, K = rows, a.gemm_n or 3 * D, D
        x, w = rn(M, K), rn(N, K)
        flops = 2.0 * M * N * K
        if op == "gemm_tc":
            return (lambda: E.gemm_tc(x, w)), flops, 0
        if op == "gemm_cublas":
            return (lambda: torch.matmul(x, w.t())), flops, 0
        # fused prefetch of a 16M-parameter layer gathered from 8 emulated owners on this GPU
        unit = 16 << 20
        bufs = [rn(unit) for _ in range(8)]
        ptrs = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device=dev)
        shard = unit // 8
        return (lambda: E.gemm_gather_tc(x, w, bufs[0], ptrs, 0, unit, shard, 0, False)), flops, 0
    raise ValueError(op)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Time the extension's kernels on the training shapes")
    add = p.add_argument
    add("--op", default="all", choices=("all",) + OPS)
    add("--batch", type=int, default=2)
    add("--seq", type=int, default=4096)
    add("--heads", type=int, default=12)
    add("--head-dim", type=int, default=64)
    add("--window", type=int, default=512)
    add("--persistent", type=int, default=4)
    add("--ffn-mult", type=float, default=4.0)
    add("--vocab", type=int, default=32000)
    add("--gemm-n", type=int, default=0, help="GEMM N (default 3 x heads x head_dim)")
    add("--warmup", type=int, default=3)
    add("--iters", type=int, default=10)
    add("--no-flush", action="store_true")
    add("--peak-tflops", type=float, default=None, help="bf16 GEMM burst peak (default: the measured one)")
    add("--peak-gbs", type=float, default=None, help="HBM copy peak (default: the measured one)")
    a = p.parse_args(argv)
    from ..utils.perf import measured_peaks

    peaks = measured_peaks()
    if a.peak_tflops is None:
        a.peak_tflops = peaks["bf16_tflops"]
    if getattr(a, "peak_gbs", 0) is None:
        a.peak_gbs = peaks["hbm_gbs"]
    flush = None if a.no_flush else torch.empty(64 << 20, device="cuda", dtype=torch.float32)
    for op in (OPS if a.op == "all" else (a.op,)):
        fn, flops, nbytes = build(op, a)
        ms = time_op(fn, a.warmup, a.iters, flush)
        rec = {"op": op, "ms": round(ms, 4), "batch": a.batch, "seq": a.seq}
        if flops:
            tf = flops / ms / 1e9
            rec.update(tflops=round(tf, 1), frac_of_measured_peak=round(tf / a.peak_tflops, 3))
        if nbytes:
            gbs = nbytes / ms / 1e6
            rec.update(gbs=round(gbs, 1), frac_of_measured_peak=round(gbs / a.peak_gbs, 3))
        print(json.dumps(rec), flush=True)
    from ..ops import _ext

    status = int(_ext.ext().kernel_error_status(0, True))
    print(json.dumps({"kernel_error_status": status}))
    if status:
        raise SystemExit(f"a kernel reported error status {status}")


if __name__ == "__main__":
    main()
