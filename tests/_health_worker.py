"""One rank of the failure-detection test (tests/test_health.py); run as a module.

    python -m tests._health_worker RANK WORLD PORT MODE OUT_DIR

CPU ``gloo`` ranks step a tiny all-reduce loop with a heartbeat check before
every step.  The last rank drops out after its third step (between steps):
``leave`` announces it, ``silent`` just stops.  Each surviving rank records
whether and how it detected the loss, and how long it took.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist

from titans_pytorch_b200.parallel.health import Heartbeat, RankLost, abort_process_group


def main() -> None:
    rank, world, port, mode, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=15))
    beat_store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=15))
    check_store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=15))
    hb = Heartbeat(beat_store, rank, world, interval=0.1, timeout=2.0, check_store=check_store)
    status, t_fail = "ok", None
    t0 = time.monotonic()
    try:
        for step in range(40):
            hb.check()
            x = torch.full((4,), float(rank + 1))
            dist.all_reduce(x)
            if rank == world - 1 and step == 2:
                if mode == "leave":
                    hb.leave()
                else:
                    hb.stop()
                with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
                    json.dump({"rank": rank, "status": "left"}, f)
                os._exit(0)
            if step == 2:
                t_fail = time.monotonic()
            time.sleep(0.05)
    except (RankLost, RuntimeError) as e:
        status = f"detected:{type(e).__name__}"
        abort_process_group()
    elapsed = time.monotonic() - (t_fail or t0)
    with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "status": status, "seconds_after_loss": elapsed}, f)
    hb.stop()
    os._exit(0)


if __name__ == "__main__":
    main()
