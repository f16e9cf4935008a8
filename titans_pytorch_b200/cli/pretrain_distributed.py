"""Distributed pretraining entry point (one process per GPU).

The reference launches `scripts/pretrain_distributed.py` with ``accelerate
launch`` (DDP / FSDP chosen by an Accelerate config, `:350-413`) and takes
``--grad-accum`` and ``--precision {no,fp16,bf16}`` (`:682-691`).  Here:

* the same flags are accepted (``--grad-accum``, ``--precision``, plus every
  flag of :mod:`titans_pytorch_b200.cli.pretrain`);
* ``--parallel dp|fsdp`` picks the framework's data-parallel engine (fused
  peer-memory gradient reduce-scatter + AdamW shard + all-gather over NVLink)
  or its sharded-parameter engine -- the roles of Accelerate's DDP and FSDP;
* ``--nproc N`` without a launcher environment re-executes the command under
  ``torch.distributed.run`` with N ranks on this node (rendezvous on
  127.0.0.1), as ``accelerate launch`` would;
* the ranks share a process group with a bounded timeout and a heartbeat: a
  rank that fails makes the others stop with an error; checkpoints keep one
  optimizer file per rank; evaluation losses are reduced over the ranks.

    python -m titans_pytorch_b200.cli.pretrain_distributed --nproc 8 --model mag --batch-size 8 --seq-len 4096
    torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m titans_pytorch_b200.cli.pretrain_distributed --model mag --batch-size 8 --seq-len 4096
"""

from __future__ import annotations

import os
import socket
import sys

from .pretrain import build_parser, run

PRECISION = {"no": "none", "none": "none", "fp16": "fp16", "bf16": "bf16"}


def build_distributed_parser():
    p = build_parser()
    p.description = "Distributed pretraining of a Titans model (one process per GPU)"
    p.add_argument("--grad-accum", type=int, default=None, help="alias of --gradient-accumulation-steps")
    p.add_argument("--precision", choices=sorted(PRECISION), default=None, help="alias of --mixed-precision")
    p.add_argument("--nproc", type=int, default=0,
                   help="without a launcher environment: run this many ranks on this node via torch.distributed.run")
    return p


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def relaunch_argv(argv: list[str], nproc: int, port: int) -> list[str]:
    """The torch.distributed.run command line that runs ``argv`` (minus --nproc) on ``nproc`` ranks."""
    rest, skip = [], False
    for i, a in enumerate(argv):
        if skip:
            skip = False
            continue
        if a == "--nproc":
            skip = True
            continue
        if a.startswith("--nproc="):
            continue
        rest.append(a)
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "titans_pytorch_b200.cli.pretrain_distributed",
            *rest]


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    args = build_distributed_parser().parse_args(argv)
    if args.grad_accum is not None:
        args.gradient_accumulation_steps = args.grad_accum
    if args.precision is not None:
        args.mixed_precision = PRECISION[args.precision]
    if "WORLD_SIZE" not in os.environ and args.nproc > 1:
        cmd = relaunch_argv(argv, args.nproc, _free_port())
        os.execvp(cmd[0], cmd)
    if int(os.environ.get("WORLD_SIZE", "1")) < 2:
        print("note: WORLD_SIZE < 2 -- training in one process (use --nproc N or a launcher for data parallelism)",
              file=sys.stderr)
    return run(args)


if __name__ == "__main__":
    main()
