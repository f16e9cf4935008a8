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
  written (24 B) and the local bf16 weights written (2 B), at the measured
  6537 GB/s copy rate.

The fused step's fraction is the slower of the two roofline times divided by
the measured time.
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


def main(argv=None) -> None:
    from ..parallel.ddp import FusedDPAdamW
    from ..train.optim import FusedAdamW
    from ..train.trainer import TrainStepConfig

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--params", type=float, default=244.2, help="millions of parameters")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--link-gbs", type=float, default=770.0)
    p.add_argument("--hbm-gbs", type=float, default=6537.3)
    a = p.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    w, rank = dist.get_world_size(), dist.get_rank()
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
    t_hbm = shard * 36 / (a.hbm_gbs * 1e6)                # local HBM bytes per shard element, ms
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
