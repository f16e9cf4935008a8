"""Pretraining CLI (single GPU, or one process per GPU under torchrun).

Flags follow the reference's `scripts/pretrain.py:845-963` (model shape, data
source, optimisation, checkpointing, evaluation, logging).  Under torchrun
(WORLD_SIZE > 1) the data-parallel engine is used (fused peer-memory
reduction on GPUs); :mod:`titans_pytorch_b200.cli.pretrain_distributed` is
the launcher-oriented entry point with the reference's distributed flags.

    python -m titans_pytorch_b200.cli.pretrain --model mag --dim 256 --num-layers 4 --max-steps 100
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m titans_pytorch_b200.cli.pretrain ...

Training loop duties besides the step (reference `scripts/pretrain.py:716-837`):

* every ``--log-every`` steps: the loss is read (the only per-step host sync),
  metrics go to the log / JSONL file / wandb, and the device error words of
  the bounded cross-GPU and pipeline waits are checked;
* every ``--eval-every`` steps: mean loss over ``--eval-batches`` held-out
  batches, reduced over the ranks, and ``best_model.pt`` when it improved;
* every ``--save-every`` steps: a resumable checkpoint (every rank writes its
  optimizer shard when the state is sharded; a host barrier follows);
* under torchrun, a heartbeat check before every step, so that a rank that
  left makes the others stop with an error instead of waiting forever.
"""

from __future__ import annotations

import argparse
import json
import logging
import math
import os
import time

import torch
from torch.utils.data import DataLoader, DistributedSampler, Subset

from ..config import TitansConfig
from ..models.titans import create_model
from ..train.trainer import Trainer, TrainStepConfig
from ..utils.checkpoint import load_training_checkpoint, save_training_checkpoint
from ..utils.data import CharLevelDataset, LocalHFDataset, StreamingDataset, SyntheticDataset, TextFileDataset
from ..utils.perf import enable_gradient_checkpointing
from ..utils.tokenizer import load_tokenizer

log = logging.getLogger("titans.pretrain")


def add_model_args(p: argparse.ArgumentParser) -> None:
    a = p.add_argument
    a("--model", choices=["mac", "mag", "mal", "lmm"], default="mag")
    a("--dim", type=int, default=512)
    a("--num-heads", type=int, default=8)
    a("--num-layers", type=int, default=12)
    a("--vocab-size", type=int, default=32000)
    a("--chunk-size", type=int, default=512)
    a("--window-size", type=int, default=512)
    a("--num-persistent-tokens", type=int, default=16)
    a("--num-memory-layers", type=int, default=2)
    a("--config", type=str, default=None, help="YAML/JSON with TitansConfig fields (overrides the flags)")


def add_data_args(p: argparse.ArgumentParser) -> None:
    a = p.add_argument
    a("--dataset", type=str, default=None)
    a("--dataset-subset", type=str, default=None)
    a("--data", type=str, default=None, help="local text file")
    a("--local-dataset", type=str, default=None, help="pre-tokenized dataset directory")
    a("--tokenizer", type=str, default=None)
    a("--seq-len", type=int, default=512)
    a("--num-workers", type=int, default=2)
    a("--synthetic-samples", type=int, default=10000)


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Pretrain a Titans model")
    add_model_args(p)
    add_data_args(p)
    a = p.add_argument
    a("--epochs", type=int, default=1)
    a("--max-steps", type=int, default=-1)
    a("--batch-size", type=int, default=8)
    a("--gradient-accumulation-steps", type=int, default=1)
    a("--lr", type=float, default=4e-4)
    a("--weight-decay", type=float, default=0.1)
    a("--grad-clip", type=float, default=1.0)
    a("--warmup-ratio", type=float, default=0.03)
    a("--parallel", choices=["dp", "fsdp", "cp", "pp"], default="dp",
      help="under torchrun: dp = replicated weights with the optimizer state sharded; fsdp = parameters "
           "sharded per block, all-gathered in the forward; cp = context parallel (MAG/MAL/LMM): every "
           "sequence split over the ranks, halos exchanged, memory updates averaged; pp = pipeline "
           "(MAC): layers split into stages, one per rank, segments as micro-batches")
    a("--mixed-precision", choices=["none", "fp16", "bf16"], default="bf16",
      help="bf16 (default) or none (fp32); fp16 is rejected: the kernels compute in bf16")
    a("--checkpoint-dir", type=str, default="checkpoints")
    a("--save-every", type=int, default=1000)
    a("--eval-every", type=int, default=500, help="evaluate every N optimizer steps (0: never)")
    a("--eval-batches", type=int, default=16, help="held-out batches per evaluation (per rank)")
    a("--resume", type=str, default=None)
    a("--log-every", type=int, default=10)
    a("--metrics-file", type=str, default=None, help="append JSON lines of metrics here")
    a("--wandb", action="store_true")
    a("--wandb-project", type=str, default="titans")
    a("--wandb-run-name", type=str, default=None)
    a("--seed", type=int, default=42)
    a("--torch-compile", action="store_true",
      help="capture the whole training step in a CUDA graph and replay it (the B200 counterpart of "
           "torch.compile's reduce-overhead mode; needs a CUDA device and no gradient accumulation)")
    a("--compile-mode", type=str, default="reduce-overhead",
      help="with --torch-compile: reduce-overhead / max-autotune / default all mean CUDA-graph replay")
    a("--gradient-checkpointing", action="store_true")
    a("--cp-size", type=int, default=0,
      help="--parallel cp: ranks per context-parallel group (default: all ranks); the groups are data-parallel "
           "replicas of each other")
    a("--wavefront", type=int, default=0,
      help="MAC: run the (layer, segment) loop as a wavefront on this many CUDA streams (0 = sequential; "
           "not with --parallel fsdp)")
    a("--heartbeat-timeout", type=float, default=60.0,
      help="under torchrun: seconds without a peer's heartbeat before this rank stops with an error")
    a("--dist-timeout", type=float, default=600.0, help="process-group timeout (seconds)")
    return p


def build_dataset(args, vocab_size):
    tok = load_tokenizer(args.tokenizer, vocab_size) if args.tokenizer else None
    if args.local_dataset:
        return LocalHFDataset(args.local_dataset, args.seq_len)
    if args.dataset:
        return StreamingDataset(args.dataset, tok or load_tokenizer(None, vocab_size), args.seq_len,
                                subset=args.dataset_subset)
    if args.data:
        return TextFileDataset(args.data, tok, args.seq_len) if tok else CharLevelDataset(args.data, vocab_size,
                                                                                           args.seq_len)
    return SyntheticDataset(vocab_size, args.seq_len, args.synthetic_samples, seed=args.seed)


def split_eval(args, ds, vocab_size):
    """(train, eval) datasets.  Synthetic data gets an independent eval set
    (another seed); map-style datasets hold out their last 1 % (at least
    ``eval_batches * batch_size`` samples); streams get no eval set."""
    need = max(1, args.eval_batches) * args.batch_size
    if args.eval_every <= 0:
        return ds, None
    if isinstance(ds, SyntheticDataset):
        return ds, SyntheticDataset(vocab_size, args.seq_len, need, seed=args.seed + 1)
    if hasattr(ds, "__len__") and len(ds) > 2 * need:
        n = len(ds)
        k = max(need, n // 100)
        return Subset(ds, range(0, n - k)), Subset(ds, range(n - k, n))
    log.warning("no held-out split for this dataset: --eval-every disabled")
    return ds, None


def setup_distributed(args, device):
    """Process group (NCCL on GPUs, gloo otherwise) with a bounded timeout, the
    data-parallel engine and a heartbeat; (engine, heartbeat) or (None, None)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return None, None
    import datetime

    import torch.distributed as dist

    from ..parallel.ddp import DataParallelEngine
    from ..parallel.fsdp import FullyShardedEngine
    from ..parallel.health import Heartbeat, store_client

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl" if device.type == "cuda" else "gloo",
                            timeout=datetime.timedelta(seconds=args.dist_timeout))
    if args.parallel == "pp":
        from ..parallel.pipeline import PipelineEngine

        engine = PipelineEngine()
    else:
        engine = FullyShardedEngine() if args.parallel == "fsdp" else DataParallelEngine()
    hb = None
    beat, check = store_client(), store_client()
    if beat is not None and check is not None:
        hb = Heartbeat(beat, dist.get_rank(), world, interval=1.0, timeout=args.heartbeat_timeout, check_store=check)
    return engine, hb


def run(args) -> dict:
    """The training loop shared by both pretraining entry points; returns the final metrics."""
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    if args.mixed_precision == "fp16":
        raise SystemExit("--mixed-precision fp16 is not supported: the sm_100a kernels compute in bf16 "
                         "(use bf16, the default, or none for fp32)")
    world, rank, local = (int(os.environ.get(k, d)) for k, d in (("WORLD_SIZE", 1), ("RANK", 0), ("LOCAL_RANK", 0)))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    engine, hb = setup_distributed(args, device)
    from ..parallel.health import DeviceWaitTimeout, RankLost, abort_process_group

    torch.manual_seed(args.seed)
    fields = dict(dim=args.dim, num_heads=args.num_heads, num_layers=args.num_layers, vocab_size=args.vocab_size,
                  chunk_size=args.chunk_size, window_size=args.window_size,
                  num_persistent_tokens=args.num_persistent_tokens, num_memory_layers=args.num_memory_layers,
                  dropout=0.0, max_seq_len=max(args.seq_len, 512))
    if args.config:
        fields.update(TitansConfig.from_file(args.config).to_dict())
    cfg = TitansConfig(**fields)
    model = create_model(args.model, cfg)
    cp = None
    cps = 1
    if args.parallel == "cp" and world > 1:
        import torch.distributed as dist

        from ..parallel.context import enable_context_parallel

        cps = args.cp_size or world
        if world % cps or args.seq_len % cps:
            raise SystemExit(f"--parallel cp: --cp-size {cps} must divide the {world} ranks and --seq-len "
                             f"{args.seq_len}")
        # every rank creates every group, in the same order
        groups = [dist.new_group(list(range(g * cps, (g + 1) * cps))) for g in range(world // cps)]
        cp = enable_context_parallel(model, groups[rank // cps] if cps < world else None)
    if args.gradient_checkpointing:
        enable_gradient_checkpointing(model)
    if args.wavefront > 1 and args.model == "mac" and device.type == "cuda":
        from ..utils.perf import enable_wavefront

        enable_wavefront(model, args.wavefront)
    ds, eval_ds = split_eval(args, build_dataset(args, cfg.vocab_size), cfg.vocab_size)
    # context parallel: every rank reads the same whole sequences and keeps its shard of them;
    # pipeline: every rank reads the same batches (stage 0 embeds them, the last stage scores them)
    pp = args.parallel == "pp" and world > 1
    if pp and args.model != "mac":
        raise SystemExit("--parallel pp is for --model mac")
    dworld, drank = (1, 0) if pp else ((world // cps, rank // cps) if cp is not None else (world, rank))
    sampler = DistributedSampler(ds, dworld, drank, shuffle=True, seed=args.seed) if (
        world > 1 and hasattr(ds, "__len__")) else None
    loader = DataLoader(ds, batch_size=args.batch_size, shuffle=(sampler is None and hasattr(ds, "__len__")),
                        sampler=sampler, num_workers=args.num_workers, pin_memory=device.type == "cuda",
                        drop_last=True)
    eval_loader = None
    if eval_ds is not None:
        es = DistributedSampler(eval_ds, dworld, drank, shuffle=False) if world > 1 else None
        eval_loader = DataLoader(eval_ds, batch_size=args.batch_size, sampler=es, shuffle=False, drop_last=True,
                                 num_workers=0, pin_memory=device.type == "cuda")
    if cp is not None:
        from ..parallel.context import ShardedLoader

        loader = ShardedLoader(loader, cp)
        eval_loader = ShardedLoader(eval_loader, cp) if eval_loader is not None else None
    steps_per_epoch = len(loader) // args.gradient_accumulation_steps if hasattr(ds, "__len__") else 10 ** 9
    total = args.max_steps if args.max_steps > 0 else steps_per_epoch * args.epochs
    dtype = {"bf16": torch.bfloat16, "none": torch.float32}[args.mixed_precision]
    graph = False
    if args.torch_compile:
        graph = device.type == "cuda" and args.gradient_accumulation_steps == 1 and cp is None and not pp
        log.info("--torch-compile (%s): %s", args.compile_mode,
                 "whole-step CUDA-graph capture and replay" if graph else
                 "no CUDA graph (needs a CUDA device, no gradient accumulation and no context "
                 "parallelism); running eagerly")
    tr = Trainer(model, TrainStepConfig(lr=args.lr, weight_decay=args.weight_decay, grad_clip=args.grad_clip,
                                        warmup_steps=int(total * args.warmup_ratio), total_steps=total,
                                        gradient_accumulation_steps=args.gradient_accumulation_steps, dtype=dtype,
                                        cuda_graph=graph),
                 device=device, engine=engine)
    start_epoch, best, skip = 0, float("inf"), 0
    if args.resume:
        ck = load_training_checkpoint(args.resume, tr, rank=rank, world=world)
        tr.global_step = int(ck.get("global_step", 0))
        skip = int(ck.get("data_position") or 0)  # micro-batches of the epoch already trained on
        start_epoch = int(ck.get("epoch", 0))
        best = float(ck.get("best_val_loss", best))
        log.info("resumed from %s at step %d", args.resume, tr.global_step)
    wb = None
    if args.wandb and rank == 0:
        try:
            import wandb

            wb = wandb.init(project=args.wandb_project, name=args.wandb_run_name, config=vars(args))
        except Exception as e:  # pragma: no cover
            log.warning("wandb unavailable: %s", e)

    def emit(m: dict) -> None:
        if rank != 0:
            return
        log.info(json.dumps(m))
        if args.metrics_file:
            with open(args.metrics_file, "a", encoding="utf-8") as f:
                f.write(json.dumps(m) + "\n")
        if wb is not None:
            wb.log(m, step=tr.global_step)

    def save(name: str, epoch: int, position: int | None) -> None:
        save_training_checkpoint(os.path.join(args.checkpoint_dir, name), tr, rank=rank, world=world,
                                 global_step=tr.global_step, epoch=epoch, best_val_loss=best,
                                 model_type=args.model, tokenizer_name=args.tokenizer, train_config=vars(args),
                                 data_position=position)

    tokens_per_step = args.batch_size * args.seq_len * dworld * args.gradient_accumulation_steps
    t_last, s_last = time.perf_counter(), tr.global_step
    last = {}
    done = False
    epoch = start_epoch
    try:
        for epoch in range(start_epoch, args.epochs if args.max_steps <= 0 else 10 ** 9):
            if sampler is not None:
                sampler.set_epoch(epoch)
            position = 0
            for batch in loader:
                if skip:  # resuming inside this epoch: its first micro-batches were already trained on
                    skip -= 1
                    position += 1
                    continue
                position += 1
                if hb is not None:
                    hb.check()  # between steps: a lost peer stops this rank before its next launch
                loss = tr.train_step(batch)
                boundary = tr._micro % args.gradient_accumulation_steps == 0 or tr.cfg.cuda_graph
                step = tr.global_step
                if step and boundary and step % args.log_every == 0:
                    lv = float(loss)
                    tr.check_errors()
                    dt = time.perf_counter() - t_last
                    tps = tokens_per_step * (step - s_last) / max(dt, 1e-9)
                    t_last, s_last = time.perf_counter(), step
                    last = {"train/loss": lv, "train/ppl": math.exp(min(lv, 20)),
                            "train/lr": tr.optimizer.param_groups[0]["lr"], "train/tokens_per_s": tps, "step": step}
                    emit(last)
                if eval_loader is not None and step and boundary and step % args.eval_every == 0:
                    ev = tr.evaluate(eval_loader, max_batches=args.eval_batches)
                    emit({"val/loss": ev["val_loss"], "val/ppl": ev["val_ppl"], "step": step})
                    last.update({"val/loss": ev["val_loss"]})
                    if ev["val_loss"] < best:
                        best = ev["val_loss"]
                        save("best_model.pt", epoch, position)
                if args.save_every > 0 and step and boundary and step % args.save_every == 0:
                    tr.check_errors()
                    save(f"step_{step}.pt", epoch, position)
                if step >= total:
                    done = True
                    break
            if done:
                break
        tr.check_errors()
        save("final_model.pt", epoch, None)
    except (RankLost, DeviceWaitTimeout) as e:
        log.error("stopping: %s", e)
        if hb is not None:
            hb.stop()
        abort_process_group()
        raise
    if hb is not None:
        hb.stop()
    if world > 1:
        import torch.distributed as dist

        tr._graph = None  # a captured step holding NCCL work goes before the group
        dist.destroy_process_group()
    return last


def main(argv=None) -> dict:
    return run(build_parser().parse_args(argv))


if __name__ == "__main__":
    main()
