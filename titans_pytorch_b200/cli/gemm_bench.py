"""tcgen05 GEMM (csrc/gemm_sm100.cu) against cuBLAS on the training step's GEMM shapes.

    python -m titans_pytorch_b200.cli.gemm_bench [--tokens 32768] [--dim 768] [--only NAME]
    python -m titans_pytorch_b200.cli.gemm_bench --census mag170m

``--census CONFIG`` records every GEMM one training step of that workload
(the model and batch of ``bench.py``) issues -- layout, M, N, K, fused
epilogue, split-K count -- and times each distinct one on its own (same
shapes and epilogue on fresh random tensors), with the count per step and
the share of the step's GEMM time.

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
    from ..utils.perf import measured_peaks

    return measured_peaks()["bf16_tflops"]


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
    ap.add_argument("--census", default="", help="workload name from bench.py (e.g. mag170m)")
    a = ap.parse_args(argv)
    if a.census:
        census(a)
        return

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
    gu_saved = rn(T, 2 * Fd)  # the [g | u] buffer the SwiGLU forward saves
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
        "mem_act": (2 * T * D * Fd, lambda: G.mm_act(x, wd.t().contiguous() if False else wgu[:Fd], "silu"),
                    lambda: E.act_inplace(torch.matmul(x, wgu[:Fd].t()), hf, "silu")),
        "mem_act_grad": (2 * T * D * Fd, lambda: G.mm_act_grad(dyd, wd, hf, "silu"),
                         lambda: E.act_grad_mul(torch.matmul(dyd, wd), hf, "silu")),
        "mem_err": (2 * T * Fd * D, lambda: G.mm_err(hf, wd, dyd, 1e-3),
                    lambda: E.scaled_err(torch.matmul(hf, wd.t()), dyd, 1e-3)),
        "ffn_swiglu_bwd": (2 * T * D * Fd, lambda: G.swiglu_dgrad(dyd, wd, gu_saved),
                           lambda: E.swiglu_bwd(torch.matmul(dyd, wd), gu_saved)),
        "ffn_down_resid": (2 * T * Fd * D, lambda: G.mm_tn(hf, wd, mode="resid", r=dyd),
                           lambda: torch.matmul(hf, wd.t()).add_(dyd)),
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


def census(a) -> None:
    """Time every distinct GEMM of one training step of a bench.py workload."""
    import collections
    import sys

    from ..ops import _ext
    from ..ops import gemm as G

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, root)
    import bench

    from .. import TitansConfig, create_model
    from ..train.trainer import Trainer, TrainStepConfig
    from ..utils.perf import enable_gradient_checkpointing

    cfg = bench.CONFIGS[a.census]
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    model = create_model(cfg["model"], TitansConfig(**cfg["fields"]))
    if cfg["ckpt"]:
        enable_gradient_checkpointing(model)
    tr = Trainer(model, TrainStepConfig(lr=bench.LR), device=dev)
    ids = torch.randint(0, cfg["fields"]["vocab_size"], (cfg["micro_batch"], cfg["seq"] + 1), device=dev)
    batch = {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous()}
    tr.train_step(batch)
    torch.cuda.synchronize()
    calls = collections.Counter()
    orig = G._run

    def rec(A, a_mn, B, b_mn, M, N, K, mode, c, r=None, c2=None, r2=None, gates=None, scale=1.0, act="silu",
            ffn_f=0, splits=0):
        calls[(bool(a_mn), bool(b_mn), int(M), int(N), int(K), mode, int(ffn_f), int(splits),
               str(c.dtype).replace("torch.", ""))] += 1
        return orig(A, a_mn, B, b_mn, M, N, K, mode, c, r, c2, r2, gates, scale, act, ffn_f, splits)

    G._run = rec
    try:
        tr.train_step(batch)
        torch.cuda.synchronize()
    finally:
        G._run = orig
    del tr, model
    torch.cuda.empty_cache()
    E = _ext.ext()
    flush = torch.empty(64 * 1024 * 1024, device=dev, dtype=torch.float32)
    peak = peak_tflops()
    rows, total = [], 0.0
    for (a_mn, b_mn, M, N, K, mode, ffn_f, splits, cdt), n in calls.items():
        def rn(*s):
            return (torch.randn(*s, device=dev) * 0.05).to(torch.bfloat16)

        A = rn(K, M) if a_mn else rn(M, K)
        B = rn(K, N) if b_mn else rn(N, K)
        odt = torch.float32 if cdt == "float32" else torch.bfloat16
        ccols = ffn_f if mode == "swiglu" else (2 * N if mode == "swiglu_bwd" else N)
        C = torch.zeros(M, ccols, device=dev, dtype=odt)
        R = torch.zeros(M, 2 * N if mode == "swiglu_bwd" else N, device=dev, dtype=odt)
        C2 = torch.zeros(M, 2 * ffn_f if mode == "swiglu" else N, device=dev, dtype=odt)
        R2 = torch.zeros(M, N, device=dev, dtype=odt)
        gates = torch.tensor([0.1, 0.01, 0.9], device=dev)
        E.kernel_error_status(0, True)
        t = timeit(lambda: G._run(A, a_mn, B, b_mn, M, N, K, mode, C, R, C2, R2, gates, 1.0, "silu", ffn_f, splits),
                   3, a.iters, flush)
        flops = 2.0 * M * N * K
        total += t * n
        rows.append({"layout": ("mn" if a_mn else "k") + "/" + ("mn" if b_mn else "k"), "M": M, "N": N, "K": K,
                     "mode": mode, "splits_arg": splits, "per_step": n, "ms": round(t, 4),
                     "tflops": round(flops / t / 1e9, 1), "frac_of_measured_peak": round(flops / t / 1e9 / peak, 3),
                     "err": E.kernel_error_status(0, True)})
    rows.sort(key=lambda r: -r["ms"] * r["per_step"])
    for r in rows:
        r["share"] = round(r["ms"] * r["per_step"] / total, 3)
        print(json.dumps(r))
    print(json.dumps({"census": a.census, "gemm_ms_per_step": round(total, 3), "distinct": len(rows)}))


if __name__ == "__main__":
    main()
