"""Per-step kernel-time breakdown of a training step: own kernels vs libraries vs ATen.

    python -m titans_pytorch_b200.cli.step_profile [--config mag170m] [--steps 2] [--top 25]

Builds the same model/trainer as ``bench.py`` (synthetic token ids, random
init), runs warm-up steps eagerly (no CUDA graph, so every launch is a
separate profiler record), then records ``--steps`` steps with the PyTorch
profiler's CUDA activity (CUPTI kernel records).  Each kernel is classified:

* ``own``   : this framework's sm_100a kernels (namespace ``tb::``)
* ``cublas``: cuBLAS / cuBLASLt GEMMs (``nvjet``, ``cublas``, ``gemm``/``cutlass`` names)
* ``nccl``  : NCCL collectives
* ``aten``  : PyTorch's own CUDA kernels (``at::native`` and friends)
* ``other`` : anything else

Output: one JSON line with per-class device time per step (ms), its share of
the summed kernel time, the launch count per step, and the ``--top`` kernels
by time.  The profiler serialises nothing and adds no device work, but
absolute times under a profiler are not bench numbers; use the shares (and
``bench.py`` for throughput).
"""

from __future__ import annotations

import argparse
import collections
import json
import os
import sys

import torch


def classify(name: str) -> str:
    low = name.lower()
    if "tb::" in name:
        return "own"
    if "nccl" in low:
        return "nccl"
    if "nvjet" in low or "cublas" in low or "gemm" in low or "cutlass" in low or "sm100_xmma" in low:
        return "cublas"
    if "at::" in name or "at_cuda_detail" in name or "elementwise" in low or "reduce_kernel" in low:
        return "aten"
    return "other"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="mag170m")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--top", type=int, default=25)
    ap.add_argument("--batch", type=int, default=0, help="micro-batch override (0: the config's)")
    ap.add_argument("--out", default="", help="also write the JSON to this file")
    a = ap.parse_args(argv)

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, root)
    import bench  # the training workload definitions live with the benchmark

    from torch.profiler import ProfilerActivity, profile

    from titans_pytorch_b200 import TitansConfig, create_model
    from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig
    from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

    cfg = bench.CONFIGS[a.config]
    fields, seq, mb = cfg["fields"], cfg["seq"], a.batch or cfg["micro_batch"]
    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    model = create_model(cfg["model"], TitansConfig(**fields))
    if cfg["ckpt"]:
        enable_gradient_checkpointing(model)
    tr = Trainer(model, TrainStepConfig(lr=bench.LR, betas=bench.BETAS, weight_decay=bench.WD,
                                        grad_clip=bench.CLIP), device=dev)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, fields["vocab_size"], (mb, seq + 1), generator=g).to(dev)
    batch = {"input_ids": ids[:, :-1].contiguous(), "labels": ids[:, 1:].contiguous()}
    for _ in range(a.warmup):
        tr.train_step(batch)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            tr.train_step(batch)
        torch.cuda.synchronize()

    per_class = collections.Counter()
    launches = collections.Counter()
    per_kernel = collections.Counter()
    count_kernel = collections.Counter()
    for e in prof.events():
        if e.device_type.name != "CUDA":
            continue
        n = e.name
        if "memcpy" in n.lower() or "memset" in n.lower():
            cls = "copy"
        else:
            cls = classify(n)
        us = e.device_time if hasattr(e, "device_time") else e.cuda_time
        per_class[cls] += us
        launches[cls] += 1
        per_kernel[(cls, n)] += us
        count_kernel[(cls, n)] += 1
    total = sum(per_class.values()) or 1.0
    res = {
        "config": a.config, "micro_batch": mb, "seq": seq, "steps": a.steps,
        "kernel_ms_per_step": total / 1000 / a.steps,
        "classes": {c: {"ms_per_step": v / 1000 / a.steps, "share": v / total, "launches_per_step": launches[c] / a.steps}
                    for c, v in per_class.most_common()},
        "top": [{"class": c, "kernel": n[:160], "ms_per_step": v / 1000 / a.steps,
                 "launches_per_step": count_kernel[(c, n)] / a.steps, "share": v / total}
                for (c, n), v in per_kernel.most_common(a.top)],
    }
    line = json.dumps(res)
    print(line)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")


if __name__ == "__main__":
    main()
