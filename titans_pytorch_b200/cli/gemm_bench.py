"""tcgen05 GEMM (csrc/gemm_sm100.cu) against cuBLAS on the training step's GEMM shapes.

    python -m titans_pytorch_b200.cli.gemm_bench [--tokens 32768] [--dim 768] [--only NAME]

Shapes are the TitansMAG training step's (tokens = micro-batch x sequence):
forward (x W^T), input gradient (dy W) and weight gradient (dy^T x, split-K
over the tokens) of the q|k|v, output, FFN and head projections, plus the
fused SwiGLU forward.  Each GEMM is timed with CUDA events after warm-up,
with an L2 flush (a 256 MB write) between timed launches outside the events;
the median of ``--iters`` launches is reported with TFLOP/s and the fraction
of the measured bf16 peak (``MEASURED_PEAKS.json``: the burst figure).
cuBLAS runs the same product through ``torch.matmul`` (with ``out=`` /
``addmm_`` for the accumulating weight gradient).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

import torch


def peak_tflops() -> float:
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def timeit(fn, warmup: int, iters: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.fill_(1.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return statistics.median(ts)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--ffn", type=int, default=3072)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="")
    a = ap.parse_args(argv)

    from ..ops import _ext
    from ..ops import gemm as G

    E = _ext.ext()
    dev = torch.device("cuda")
    T, D, Fd, V = a.tokens, a.dim, a.ffn, a.vocab
    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*s):
        return (torch.randn(*s, device=dev, generator=g) * 0.05).to(torch.bfloat16)

    flush = torch.empty(64 * 1024 * 1024, device=dev, dtype=torch.float32)
    peak = peak_tflops()
    x, dy3, w3 = rn(T, D), rn(T, 3 * D), rn(3 * D, D)
    wgu, wd, hf, dyd = rn(2 * Fd, D), rn(D, Fd), rn(T, Fd), rn(T, D)
    wh, dyv = rn(V, D), rn(T, V)
    gw3, gwd = torch.zeros(3 * D, D, device=dev, dtype=torch.bfloat16), torch.zeros(D, Fd, device=dev,
                                                                                   dtype=torch.bfloat16)
    out3 = torch.empty(T, 3 * D, device=dev, dtype=torch.bfloat16)
    cases = {
        # name: (flops, ours, cublas)
        "qkv_fwd": (2 * T * D * 3 * D, lambda: G.mm_tn(x, w3, out=out3), lambda: torch.matmul(x, w3.t(), out=out3)),
        "qkv_dgrad": (2 * T * D * 3 * D, lambda: G.mm_nn(dy3, w3), lambda: torch.matmul(dy3, w3)),
        "qkv_wgrad_acc": (2 * T * D * 3 * D, lambda: G.mm_wgrad(dy3, x, out=gw3, accumulate=True),
                          lambda: gw3.addmm_(dy3.t(), x)),
        "ffn_gateup_swiglu": (2 * T * D * 2 * Fd, lambda: G.swiglu_fwd(x, wgu),
                              lambda: E.swiglu_fwd(torch.matmul(x, wgu.t()))),
        "ffn_gateup_gemm_only": (2 * T * D * 2 * Fd, lambda: G.mm_tn(x, wgu), lambda: torch.matmul(x, wgu.t())),
        "ffn_down_fwd": (2 * T * Fd * D, lambda: G.mm_tn(hf, wd), lambda: torch.matmul(hf, wd.t())),
        "ffn_down_dgrad": (2 * T * Fd * D, lambda: G.mm_nn(dyd, wd), lambda: torch.matmul(dyd, wd)),
        "ffn_down_wgrad_acc": (2 * T * Fd * D, lambda: G.mm_wgrad(dyd, hf, out=gwd, accumulate=True),
                               lambda: gwd.addmm_(dyd.t(), hf)),
        "out_proj_fwd": (2 * T * D * D, lambda: G.mm_tn(x, w3[:D]), lambda: torch.matmul(x, w3[:D].t())),
        "head_fwd": (2 * T * D * V, lambda: G.mm_tn(x, wh), lambda: torch.matmul(x, wh.t())),
        "head_dgrad": (2 * T * D * V, lambda: G.mm_nn(dyv, wh), lambda: torch.matmul(dyv, wh)),
    }
    for name, (flops, ours, cub) in cases.items():
        if a.only and a.only not in name:
            continue
        E.kernel_error_status(0, True)
        t_ours = timeit(ours, a.warmup, a.iters, flush)
        err = E.kernel_error_status(0, True)
        t_cub = timeit(cub, a.warmup, a.iters, flush)
        print(json.dumps({
            "gemm": name, "tokens": T, "ours_ms": round(t_ours, 4), "cublas_ms": round(t_cub, 4),
            "ours_tflops": round(flops / t_ours / 1e9, 1), "cublas_tflops": round(flops / t_cub / 1e9, 1),
            "ours_frac_of_measured_peak": round(flops / t_ours / 1e9 / peak, 3),
            "cublas_frac_of_measured_peak": round(flops / t_cub / 1e9 / peak, 3),
            "speedup_vs_cublas": round(t_cub / t_ours, 3), "kernel_error_status": err}))


if __name__ == "__main__":
    main()
