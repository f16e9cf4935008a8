"""Context-parallel training throughput: one long sequence split over the ranks.

    python -m titans_pytorch_b200.cli.cp_bench                                  # 1 GPU
    torchrun --nnodes 1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m titans_pytorch_b200.cli.cp_bench --seq-len 65536

Model: TitansMAG with the ~170M training architecture (dim 768, 12 layers, 12
heads, window 512, L_M = 2, vocab 32000), random weights, synthetic token ids;
batch ``--batch`` sequences of ``--seq-len`` tokens per step.  With N ranks every
sequence is split into N shards (:mod:`titans_pytorch_b200.parallel.context`);
the parameters' gradients are averaged by the data-parallel engine, so the
total work per step is fixed as N grows (strong scaling).  Each step is an
eager forward + backward + AdamW through ``Trainer.train_step``.

Timing: ``--warmup`` untimed steps, then ``--steps`` steps bracketed by a
barrier and a device synchronisation, CUDA events on each rank, the maximum
over ranks.  One JSON line: tokens/s over the whole job.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch

FIELDS = dict(vocab_size=32000, dim=768, num_layers=12, num_heads=12, window_size=512, chunk_size=512,
              num_memory_layers=2, memory_hidden_mult=4.0, ffn_mult=4.0, num_persistent_tokens=16,
              dropout=0.0, init_std=0.02)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=FIELDS["num_layers"])
    args = ap.parse_args(argv)

    import torch.distributed as dist

    from .. import TitansConfig, create_model
    from ..parallel.context import enable_context_parallel, shard_batch
    from ..train.trainer import Trainer, TrainStepConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    engine = None
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        from ..parallel.ddp import DataParallelEngine

        engine = DataParallelEngine()
    torch.manual_seed(0)
    model = create_model("mag", TitansConfig(**{**FIELDS, "num_layers": args.layers,
                                                "max_seq_len": args.seq_len}))
    shard = enable_context_parallel(model) if world > 1 else None
    tr = Trainer(model, TrainStepConfig(lr=4e-4, cuda_graph=False), device=torch.device("cuda", local),
                 engine=engine)
    g = torch.Generator().manual_seed(1)
    data = torch.randint(0, FIELDS["vocab_size"], (args.batch, args.seq_len + 1), generator=g)
    batch = {"input_ids": data[:, :-1], "labels": data[:, 1:]}
    if shard is not None:
        batch = shard_batch(batch, shard)
    batch = {k: v.contiguous().cuda() for k, v in batch.items()}

    def sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        tr.train_step(batch)
    sync()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        loss = tr.train_step(batch)
    t1.record()
    sync()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens = args.batch * args.seq_len
    out = {"metric": "cp_train_tokens_per_s", "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
           "ms_per_step": ms, "seq_len": args.seq_len, "batch": args.batch, "layers": args.layers,
           "scaling": "strong", "loss": float(loss), "dtype": "bf16", "data": "synthetic"}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
