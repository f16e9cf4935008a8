"""Failure detection for one-process-per-GPU training (host side).

The reference has no failure handling beyond broad ``except Exception``
fallbacks (`src/titans/memory.py:319-320, 445-448`).  Here three mechanisms
turn a stuck or lost peer into an exception on every surviving rank instead
of a hang:

* **Bounded device waits.**  Every cross-GPU wait inside the kernels (the
  fused data-parallel step's barriers, the sharded engine's gathers) and every
  mbarrier wait of the tcgen05 kernels gives up after a cycle budget, records
  a code in a device error word and returns.  :func:`check_device_errors`
  reads the words (a device synchronisation) and raises
  :class:`DeviceWaitTimeout`; the training loop calls it at its log and save
  points.
* **Heartbeats.**  :class:`Heartbeat` publishes a beat counter per rank to the
  process group's key-value store from a daemon thread (so long host work such
  as a checkpoint write does not look like a dead rank), and ``check()`` --
  called between steps, before the next step's first launch -- raises
  :class:`RankLost` when a peer announced that it left, or when its beat has
  not advanced for ``timeout`` seconds (measured on this rank's monotonic
  clock, so clocks of different hosts never get compared).
* **Abort.**  :func:`abort_process_group` tears the group down so that no
  surviving rank stays blocked in a collective.

Ranks leave only between steps (no kernel or collective in flight), which is
the only way a rank may drop out of a GPU job without faulting its peers.
"""

from __future__ import annotations

import threading
import time

import torch


class DeviceWaitTimeout(RuntimeError):
    """A bounded device-side wait ran out (a peer or a pipeline stage never arrived)."""


class RankLost(RuntimeError):
    """A peer rank left the job or stopped beating."""


def check_device_errors(optimizer=None, device=None, reset: bool = True) -> None:
    """Raise :class:`DeviceWaitTimeout` if a kernel recorded a timed-out wait.

    Reads the tcgen05 kernels' error word of ``device`` and, when given, the
    optimizer's cross-GPU barrier word (``optimizer.err``).  Synchronises.
    """
    codes = []
    err = getattr(optimizer, "err", None)
    if isinstance(err, torch.Tensor) and err.numel():
        v = int(err.reshape(-1)[0].item())
        if v:
            codes.append(("cross-GPU barrier", v))
            if reset:
                err.zero_()
    if device is not None and torch.device(device).type == "cuda":
        from ..ops import _ext

        if _ext.available():
            v = int(_ext.ext().kernel_error_status(torch.device(device).index or 0, reset))
            if v:
                codes.append(("tcgen05 kernel", v))
    if codes:
        raise DeviceWaitTimeout("bounded device wait timed out: " + ", ".join(f"{w} (code {c})" for w, c in codes))


class Heartbeat:
    """Per-rank liveness through a key-value store (``torch.distributed.Store``).

    ``store``: a store client this object may use from its beat thread (give it
    its own connection, e.g. ``dist.TCPStore(host, port, is_master=False)``);
    ``check_store``: the store used by :meth:`check` in the caller's thread
    (defaults to ``store``).
    """

    PREFIX = "titans/health"

    def __init__(self, store, rank: int, world: int, interval: float = 0.5, timeout: float = 10.0,
                 check_store=None, start: bool = True) -> None:
        self.store = store
        self.check_store = check_store if check_store is not None else store
        self.rank, self.world = rank, world
        self.interval, self.timeout = float(interval), float(timeout)
        self._beats = 0
        self._stop = threading.Event()
        self._seen: dict[int, tuple[int, float]] = {}
        self._thread = None
        self._beat()
        if start:
            self._thread = threading.Thread(target=self._run, name=f"titans-heartbeat-{rank}", daemon=True)
            self._thread.start()

    def _key(self, kind: str, r: int) -> str:
        return f"{self.PREFIX}/{kind}/{r}"

    def _beat(self) -> None:
        self._beats += 1
        self.store.set(self._key("beat", self.rank), str(self._beats))

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:  # the store went away (job ending): stop beating
                return

    def check(self) -> None:
        """Raise :class:`RankLost` if a peer left or its beat is stale."""
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.check_store.check([self._key("left", r)]):
                raise RankLost(f"rank {r} left the job")
            key = self._key("beat", r)
            if not self.check_store.check([key]):
                beat = -1
            else:
                beat = int(self.check_store.get(key))
            last = self._seen.get(r)
            if last is None or beat != last[0]:
                self._seen[r] = (beat, now)
            elif now - last[1] > self.timeout:
                raise RankLost(f"rank {r} has not beaten for {now - last[1]:.1f} s")

    def leave(self) -> None:
        """Announce that this rank leaves (call between steps), then stop beating."""
        self.store.set(self._key("left", self.rank), "1")
        self.stop()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None and self._thread is not threading.current_thread():
            self._thread.join(timeout=2 * self.interval + 1)


def abort_process_group(group=None) -> None:
    """Tear the process group down after a failure (no-op without one)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return
    try:
        pg = group if group is not None else dist.distributed_c10d._get_default_group()
        abort = getattr(pg, "abort", None)
        if callable(abort):
            abort()
            return
    except Exception:
        pass
    try:
        dist.destroy_process_group(group)
    except Exception:
        pass


def store_client(timeout: float = 30.0):
    """A fresh client connection to the launcher's TCP store (MASTER_ADDR / MASTER_PORT),
    for a heartbeat thread; None when the environment does not name one."""
    import datetime
    import os

    import torch.distributed as dist

    host, port = os.environ.get("MASTER_ADDR"), os.environ.get("MASTER_PORT")
    if not host or not port:
        return None
    try:
        return dist.TCPStore(host, int(port), is_master=False, timeout=datetime.timedelta(seconds=timeout))
    except Exception:
        return None


__all__ = ["DeviceWaitTimeout", "RankLost", "check_device_errors", "Heartbeat", "abort_process_group",
           "store_client"]
