"""Distributed pretraining entry point (one process per GPU, launched with torchrun).

The reference drives DDP/FSDP through Accelerate (`scripts/pretrain_distributed.py`);
here the same flags as :mod:`titans_pytorch_b200.cli.pretrain` run under
torchrun with the framework's data-parallel engine:

    torchrun --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m titans_pytorch_b200.cli.pretrain_distributed --model mag --batch-size 8 --seq-len 4096
"""

from __future__ import annotations

import os
import sys

from .pretrain import main as _main


def main(argv=None) -> None:
    if int(os.environ.get("WORLD_SIZE", "1")) < 2:
        print("note: WORLD_SIZE < 2 -- running single-process (launch with torchrun for data parallelism)",
              file=sys.stderr)
    _main(argv)


if __name__ == "__main__":
    main()
