"""Failure detection (SURVEY 5.3 forms that fault no GPU).

* CPU gloo ranks: a rank that leaves between steps (announced, or silently)
  makes every survivor raise within a bounded time instead of hanging.
* Heartbeat logic against an in-process store.
* GPU (one device): the fused data-parallel barrier's bounded wait on a flag
  nothing sets runs out, records its code in the error word and returns; the
  host check turns that into DeviceWaitTimeout, and the device stays usable.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import time

import pytest
import torch

from titans_pytorch_b200.parallel.health import DeviceWaitTimeout, Heartbeat, RankLost, check_device_errors

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["leave", "silent"])
def test_survivors_detect_lost_rank(tmp_path, mode):
    world, port = 3, _free_port()
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    procs = [subprocess.Popen([sys.executable, "-m", "tests._health_worker", str(r), str(world), str(port), mode,
                               str(tmp_path)], cwd=ROOT, env=env) for r in range(world)]
    deadline = time.monotonic() + 90
    try:
        for p in procs:
            p.wait(timeout=max(1.0, deadline - time.monotonic()))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    res = {}
    for r in range(world):
        with open(tmp_path / f"rank{r}.json") as f:
            res[r] = json.load(f)
    assert res[world - 1]["status"] == "left"
    for r in range(world - 1):
        assert res[r]["status"].startswith("detected"), res[r]
        assert res[r]["seconds_after_loss"] < 30.0, res[r]
    if mode == "leave":  # an announced departure is seen at the next step's check
        for r in range(world - 1):
            assert res[r]["status"] == "detected:RankLost", res[r]


def test_heartbeat_stale_and_left():
    import torch.distributed as dist

    store = dist.HashStore()
    hb0 = Heartbeat(store, 0, 2, interval=0.05, timeout=0.3)
    hb1 = Heartbeat(store, 1, 2, interval=0.05, timeout=0.3)
    hb0.check()
    time.sleep(0.2)
    hb0.check()  # rank 1 beats: fine
    hb1.stop()
    hb0.check()  # records the last beat
    time.sleep(0.5)
    with pytest.raises(RankLost):
        hb0.check()
    store2 = dist.HashStore()
    a = Heartbeat(store2, 0, 2, interval=0.05, timeout=10.0)
    b = Heartbeat(store2, 1, 2, interval=0.05, timeout=10.0)
    b.leave()
    with pytest.raises(RankLost, match="left"):
        a.check()
    a.stop()
    hb0.stop()


def test_check_device_errors_cpu_word():
    class Opt:
        err = torch.tensor([0], dtype=torch.int32)

    check_device_errors(Opt())
    Opt.err[0] = 101
    with pytest.raises(DeviceWaitTimeout, match="code 101"):
        check_device_errors(Opt())
    assert int(Opt.err[0]) == 0  # reset after the report


@pytest.mark.gpu
def test_barrier_wait_runs_out_and_reports():
    """One rank of a 2-rank barrier whose peer never arrives: the bounded wait
    (short budget) sets 100 + slot in the error word and the kernel returns."""
    from titans_pytorch_b200.ops import _ext

    E = _ext.ext()
    dev = torch.device("cuda", 0)
    world, slot = 2, 1
    sig = [torch.zeros(3 * world, dtype=torch.int32, device=dev) for _ in range(world)]
    ptrs = torch.tensor([s.data_ptr() for s in sig], dtype=torch.int64, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.monotonic()
    E.comm_barrier(ptrs, slot, epoch, True, world, 0, err, 50_000_000)
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 20
    assert int(err.item()) == 100 + slot

    class Opt:
        pass

    o = Opt()
    o.err = err
    with pytest.raises(DeviceWaitTimeout, match=f"code {100 + slot}"):
        check_device_errors(o, dev)
    # the context is still usable
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2
    # a barrier whose peer did arrive completes without an error
    sig[0][slot * world + 1] = 5
    epoch.fill_(4)
    E.comm_barrier(ptrs, slot, epoch, True, world, 0, err, 50_000_000)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
