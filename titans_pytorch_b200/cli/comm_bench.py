"""Fused data-parallel step vs NCCL, device-timed (max over ranks).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m titans_pytorch_b200.cli.comm_bench --params 244.2

The workload is a flat bf16 parameter set with random gradients, 244.2 M
parameters by default (the TitansMAG ~170M model). Two arms are timed:

* fused: ``FusedDPAdamW.step``. One pass reduce-scatters the gradients by peer
  loads, publishes the norm, clips, runs AdamW on this rank's shard and
  all-gathers the new bf16 weights by peer stores, all over NVLink peer memory.
* nccl: ``dist.all_reduce`` of the bf16 gradient buffer, then the single-GPU
  fused AdamW on the full replica (the DDP + optimizer baseline).

Each is timed with CUDA events around ``--steps`` steps after ``--warmup``; the
max over ranks is reported.  Roofline of the fused step, per rank:

* NVLink: (w-1)/w of the bf16 gradient crosses in (reduce-scatter) and (w-1)/w
  of the bf16 weights crosses out (all-gather), in two phases, at 770 GB/s per
  direction (a measured peer copy on this system).
* HBM: per shard element, the local bf16 gradient read (2 B), the fp32 reduce
  buffer written and read (8 B), master weights and both moments read and
  written (24 B) and the local bf16 weights written (2 B); per element of the
  other ranks' shards, their loads of this GPU's gradient (2 B) and their
  stores of the new weights into this GPU's buffer (2 B); at the measured
  copy rate (``hbm_gbs`` of ``MEASURED_PEAKS.json``).

The fused step's fraction is the slower of the two roofline times divided by
the measured time.

``--what gather_gemm`` times the sharded-parameter forward kernel: the first
GEMM of a TitansMAG ~170M block (q|k|v projection, [8 x 4096, 768] x
[2304, 768]^T) while the next block's 18.28 M parameters (bf16, sharded over
the ranks) are all-gathered into this rank's buffer by the same kernel, peer
memory over NVLink.  Arms: the fused kernel (prefetch mode: the GEMM's weights
are local, the gather targets the next block), the same kernel in consume mode
(the weights are part of the gathered unit; tiles wait for their rows), the
GEMM alone, and the unfused baseline (cuBLAS GEMM, then NCCL
``all_gather_into_tensor`` of the shards) sequentially and overlapped on two
streams.  Roofline: the slower of 2MNK at the measured bf16 GEMM peak and the
(w-1)/w x 2 bytes x unit that must cross NVLink into this GPU at 770 GB/s.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


class _Flat(torch.nn.Module):
    def __init__(self, n: int, chunk: int = 1 << 24):
        super().__init__()
        sizes = [chunk] * (n // chunk) + ([n % chunk] if n % chunk else [])
        self.ps = torch.nn.ParameterList(torch.nn.Parameter(torch.zeros(s)) for s in sizes)


def _time(fn, warmup: int, steps: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def gather_gemm(a, w: int, rank: int) -> None:
    from ..ops._ext import ext
    from ..parallel.ddp import _PeerBuffer

    E = ext()
    M, N, K = a.gemm_m, a.gemm_n, a.gemm_k
    unit = int(a.unit_params * 1e6) // 8 * 8
    shard = -(-unit // w // 8) * 8
    g = torch.Generator(device="cuda").manual_seed(rank)
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    W = torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=g)
    buf = _PeerBuffer(unit * 2, torch.device("cuda", torch.cuda.current_device()), None, w, rank)
    flat = buf.local.view(torch.bfloat16)
    flat.copy_(torch.randn(unit, device="cuda", generator=g).to(torch.bfloat16))
    dist.barrier()
    Wu = flat[:N * K].view(N, K)  # consume mode: the GEMM's weight is the unit's first rows

    def fused():
        E.gemm_gather_tc(A, W, flat, buf.ptrs, 0, unit, shard, rank, False)

    def consume():
        E.gemm_gather_tc(A, Wu, flat, buf.ptrs, 0, unit, shard, rank, True)

    def gemm_only():
        E.gemm_tc(A, W)

    mine = flat[rank * shard:min(unit, (rank + 1) * shard)]
    gathered = torch.empty(shard * w, device="cuda", dtype=torch.bfloat16)
    piece = torch.zeros(shard, device="cuda", dtype=torch.bfloat16)
    piece[:mine.numel()].copy_(mine)
    side = torch.cuda.Stream()

    def nccl_seq():
        torch.matmul(A, W.t())
        dist.all_gather_into_tensor(gathered, piece)

    def nccl_overlap():
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            dist.all_gather_into_tensor(gathered, piece)
        torch.matmul(A, W.t())
        torch.cuda.current_stream().wait_stream(side)

    res = {name: _time(fn, a.warmup, a.steps) for name, fn in
           (("fused_prefetch", fused), ("fused_consume", consume), ("gemm_tc_alone", gemm_only),
            ("cublas_then_nccl_allgather", nccl_seq), ("cublas_nccl_allgather_overlapped", nccl_overlap))}
    st = int(E.kernel_error_status(torch.cuda.current_device(), True))
    t_gemm = 2.0 * M * N * K / (a.gemm_tflops * 1e9)
    link = (w - 1) / w * unit * 2
    t_link = link / (a.link_gbs * 1e6)
    roof = max(t_gemm, t_link)
    if rank == 0:
        print(json.dumps({"bench": "gather_gemm", "world": w, "M": M, "N": N, "K": K, "unit_params_m": a.unit_params,
                          "ms": {k: round(v, 4) for k, v in res.items()},
                          "nvlink_bytes_in_per_rank": link,
                          "roofline_ms": {"gemm": round(t_gemm, 4), "nvlink": round(t_link, 4)},
                          "frac_of_roofline": {k: round(roof / res[k], 3) for k in ("fused_prefetch", "fused_consume")},
                          "kernel_error_status": st}))
    dist.barrier()
    buf.close()


def main(argv=None) -> None:
    from ..parallel.ddp import FusedDPAdamW
    from ..train.optim import FusedAdamW
    from ..train.trainer import TrainStepConfig

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--params", type=float, default=244.2, help="millions of parameters")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--link-gbs", type=float, default=770.0)
    p.add_argument("--hbm-gbs", type=float, default=None, help="default: the measured copy rate")
    p.add_argument("--what", choices=["dp_step", "gather_gemm", "all"], default="all")
    p.add_argument("--gemm-m", type=int, default=8 * 4096)
    p.add_argument("--gemm-n", type=int, default=3 * 768)
    p.add_argument("--gemm-k", type=int, default=768)
    p.add_argument("--unit-params", type=float, default=18.284544, help="millions of parameters gathered")
    p.add_argument("--gemm-tflops", type=float, default=None, help="default: the measured bf16 GEMM burst peak")
    a = p.parse_args(argv)
    from ..utils.perf import measured_peaks

    peaks = measured_peaks()
    a.hbm_gbs = peaks["hbm_gbs"] if a.hbm_gbs is None else a.hbm_gbs
    a.gemm_tflops = peaks["bf16_tflops"] if a.gemm_tflops is None else a.gemm_tflops
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    w, rank = dist.get_world_size(), dist.get_rank()
    if a.what in ("gather_gemm", "all"):
        gather_gemm(a, w, rank)
    if a.what == "gather_gemm":
        dist.destroy_process_group()
        return
    n = int(a.params * 1e6)
    g = torch.Generator(device="cuda").manual_seed(rank)
    cfg = TrainStepConfig(lr=4e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0)

    model = _Flat(n).cuda().to(torch.bfloat16)
    fused = FusedDPAdamW(model, cfg)
    fused.space.grad.copy_(torch.randn(fused.space.grad.shape, device="cuda", generator=g) * 1e-3)
    fused.space.got = [True] * len(fused.space.params)
    ms_fused = _time(fused.step, a.warmup, a.steps)
    fused.check_errors()
    fused.close()
    del fused, model
    torch.cuda.empty_cache()

    model = _Flat(n).cuda().to(torch.bfloat16)
    opt = FusedAdamW(model.parameters(), lr=cfg.lr, betas=cfg.betas, weight_decay=cfg.weight_decay,
                     max_grad_norm=cfg.grad_clip)
    opt.space.grad.copy_(torch.randn(opt.space.grad.shape, device="cuda", generator=g) * 1e-3)
    opt.space.got = [True] * len(opt.space.params)

    def nccl_step():
        dist.all_reduce(opt.space.grad)
        opt.step()

    ms_nccl = _time(nccl_step, a.warmup, a.steps)

    shard = n / w
    link_bytes = 2 * (w - 1) / w * n * 2             # bf16 in (reduce-scatter) + bf16 out (all-gather)
    t_link = (w - 1) / w * n * 2 / (a.link_gbs * 1e6) * 2  # two phases, one direction each, ms
    t_hbm = (shard * 36 + (n - shard) * 4) / (a.hbm_gbs * 1e6)  # bytes this GPU's HBM serves, ms
    roof = max(t_link, t_hbm)
    if rank == 0:
        print(json.dumps({"bench": "fused_dp_step", "world": w, "params_m": a.params,
                          "fused_ms": round(ms_fused, 4), "nccl_allreduce_plus_adamw_ms": round(ms_nccl, 4),
                          "speedup_vs_nccl": round(ms_nccl / ms_fused, 3),
                          "nvlink_bytes_per_rank": link_bytes, "roofline_ms": {"nvlink": round(t_link, 4),
                                                                               "hbm": round(t_hbm, 4)},
                          "frac_of_roofline": round(roof / ms_fused, 3)}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
