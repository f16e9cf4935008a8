"""Pretraining CLI (single GPU, or one process per GPU under torchrun).

Flags follow the reference's `scripts/pretrain.py:845-963` (model shape, data
source, optimisation, checkpointing, logging).  Under torchrun (WORLD_SIZE > 1)
the data-parallel engine is used (fused peer-memory reduction on GPUs).

    python -m titans_pytorch_b200.cli.pretrain --model mag --dim 256 --num-layers 4 --max-steps 100
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m titans_pytorch_b200.cli.pretrain ...
"""

from __future__ import annotations

import argparse
import json
import logging
import math
import os
import time

import torch
from torch.utils.data import DataLoader, DistributedSampler

from ..config import TitansConfig
from ..models.titans import create_model
from ..train.trainer import Trainer, TrainStepConfig
from ..utils.checkpoint import load_checkpoint, save_checkpoint
from ..utils.data import CharLevelDataset, LocalHFDataset, StreamingDataset, SyntheticDataset, TextFileDataset
from ..utils.perf import enable_gradient_checkpointing
from ..utils.tokenizer import load_tokenizer

log = logging.getLogger("titans.pretrain")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="Pretrain a Titans model")
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
    a("--dataset", type=str, default=None)
    a("--dataset-subset", type=str, default=None)
    a("--data", type=str, default=None, help="local text file")
    a("--local-dataset", type=str, default=None, help="pre-tokenized dataset directory")
    a("--tokenizer", type=str, default=None)
    a("--seq-len", type=int, default=512)
    a("--epochs", type=int, default=1)
    a("--max-steps", type=int, default=-1)
    a("--batch-size", type=int, default=8)
    a("--gradient-accumulation-steps", type=int, default=1)
    a("--lr", type=float, default=4e-4)
    a("--weight-decay", type=float, default=0.1)
    a("--grad-clip", type=float, default=1.0)
    a("--warmup-ratio", type=float, default=0.03)
    a("--parallel", choices=["dp", "fsdp"], default="dp",
      help="under torchrun: dp = replicated weights with the optimizer state sharded; fsdp = parameters "
           "sharded per block, all-gathered in the forward")
    a("--mixed-precision", choices=["none", "fp16", "bf16"], default="bf16")
    a("--checkpoint-dir", type=str, default="checkpoints")
    a("--save-every", type=int, default=1000)
    a("--eval-every", type=int, default=500)
    a("--resume", type=str, default=None)
    a("--log-every", type=int, default=10)
    a("--metrics-file", type=str, default=None, help="append JSON lines of metrics here")
    a("--wandb", action="store_true")
    a("--wandb-project", type=str, default="titans")
    a("--wandb-run-name", type=str, default=None)
    a("--seed", type=int, default=42)
    a("--num-workers", type=int, default=2)
    a("--synthetic-samples", type=int, default=10000)
    a("--torch-compile", action="store_true", help="accepted for compatibility; kernels are native")
    a("--compile-mode", type=str, default="reduce-overhead")
    a("--gradient-checkpointing", action="store_true")
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


def _full_params(tr) -> None:
    """Every rank: gather parameters that are still sharded (FSDP) before rank 0 reads them."""
    mat = getattr(tr.optimizer, "materialize", None)
    if mat is not None:
        mat()


def main(argv=None) -> None:
    args = build_parser().parse_args(argv)
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    world, rank, local = (int(os.environ.get(k, d)) for k, d in (("WORLD_SIZE", 1), ("RANK", 0), ("LOCAL_RANK", 0)))
    engine = None
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if world > 1:
        import datetime

        import torch.distributed as dist

        from ..parallel.ddp import DataParallelEngine
        from ..parallel.fsdp import FullyShardedEngine

        dist.init_process_group("nccl" if device.type == "cuda" else "gloo",
                                timeout=datetime.timedelta(seconds=600))
        engine = FullyShardedEngine() if args.parallel == "fsdp" else DataParallelEngine()
    torch.manual_seed(args.seed)
    fields = dict(dim=args.dim, num_heads=args.num_heads, num_layers=args.num_layers, vocab_size=args.vocab_size,
                  chunk_size=args.chunk_size, window_size=args.window_size,
                  num_persistent_tokens=args.num_persistent_tokens, num_memory_layers=args.num_memory_layers,
                  dropout=0.0, max_seq_len=max(args.seq_len, 512))
    if args.config:
        fields.update(TitansConfig.from_file(args.config).to_dict())
    cfg = TitansConfig(**fields)
    model = create_model(args.model, cfg)
    if args.gradient_checkpointing:
        enable_gradient_checkpointing(model)
    ds = build_dataset(args, cfg.vocab_size)
    sampler = DistributedSampler(ds, world, rank, shuffle=True, seed=args.seed) if (
        world > 1 and hasattr(ds, "__len__")) else None
    loader = DataLoader(ds, batch_size=args.batch_size, shuffle=(sampler is None and hasattr(ds, "__len__")),
                        sampler=sampler, num_workers=args.num_workers, pin_memory=device.type == "cuda",
                        drop_last=True)
    steps_per_epoch = len(loader) // args.gradient_accumulation_steps if hasattr(ds, "__len__") else 10 ** 9
    total = args.max_steps if args.max_steps > 0 else steps_per_epoch * args.epochs
    dtype = {"bf16": torch.bfloat16, "fp16": torch.bfloat16, "none": torch.float32}[args.mixed_precision]
    tr = Trainer(model, TrainStepConfig(lr=args.lr, weight_decay=args.weight_decay, grad_clip=args.grad_clip,
                                        warmup_steps=int(total * args.warmup_ratio), total_steps=total,
                                        gradient_accumulation_steps=args.gradient_accumulation_steps, dtype=dtype),
                 device=device, engine=engine)
    start_epoch = 0
    if args.resume:
        ck = load_checkpoint(args.resume, tr.model, tr.optimizer, tr.scheduler)
        tr.global_step = int(ck.get("global_step", 0))
        start_epoch = int(ck.get("epoch", 0))
    wb = None
    if args.wandb and rank == 0:
        try:
            import wandb

            wb = wandb.init(project=args.wandb_project, name=args.wandb_run_name, config=vars(args))
        except Exception as e:  # pragma: no cover
            log.warning("wandb unavailable: %s", e)
    tokens_per_step = args.batch_size * args.seq_len * world * args.gradient_accumulation_steps
    t_last, s_last = time.perf_counter(), tr.global_step
    done = False
    for epoch in range(start_epoch, args.epochs if args.max_steps <= 0 else 10 ** 9):
        if sampler is not None:
            sampler.set_epoch(epoch)
        for batch in loader:
            loss = tr.train_step(batch)
            if tr.global_step and tr.global_step % args.log_every == 0 and tr._micro % args.gradient_accumulation_steps == 0:
                lv = float(loss)
                dt = time.perf_counter() - t_last
                tps = tokens_per_step * (tr.global_step - s_last) / max(dt, 1e-9)
                t_last, s_last = time.perf_counter(), tr.global_step
                m = {"train/loss": lv, "train/ppl": math.exp(min(lv, 20)),
                     "train/lr": tr.optimizer.param_groups[0]["lr"], "train/tokens_per_s": tps,
                     "step": tr.global_step}
                if rank == 0:
                    log.info(json.dumps(m))
                    if args.metrics_file:
                        with open(args.metrics_file, "a", encoding="utf-8") as f:
                            f.write(json.dumps(m) + "\n")
                    if wb is not None:
                        wb.log(m, step=tr.global_step)
            if args.save_every > 0 and tr.global_step and tr.global_step % args.save_every == 0 \
                    and tr._micro % args.gradient_accumulation_steps == 0:
                _full_params(tr)
            if rank == 0 and args.save_every > 0 and tr.global_step and tr.global_step % args.save_every == 0 \
                    and tr._micro % args.gradient_accumulation_steps == 0:
                save_checkpoint(os.path.join(args.checkpoint_dir, f"step_{tr.global_step}.pt"), tr.model,
                                tr.optimizer, tr.scheduler, global_step=tr.global_step, epoch=epoch,
                                model_type=args.model, tokenizer_name=args.tokenizer, train_config=vars(args))
            if tr.global_step >= total:
                done = True
                break
        if done:
            break
    _full_params(tr)
    if rank == 0:
        save_checkpoint(os.path.join(args.checkpoint_dir, "final_model.pt"), tr.model, tr.optimizer, tr.scheduler,
                        global_step=tr.global_step, model_type=args.model, tokenizer_name=args.tokenizer,
                        train_config=vars(args))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
