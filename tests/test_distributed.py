"""Data-parallel engine: multi-process tests (gloo ranks on CPU; NCCL + peer memory on 2 GPUs)."""

from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import titans_pytorch_b200 as T
from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig

FIELDS = dict(dim=64, num_heads=2, num_layers=2, vocab_size=128, window_size=16, chunk_size=32,
              num_persistent_tokens=4, dropout=0.0, max_seq_len=128, ffn_mult=2.0, memory_hidden_mult=2.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batches(steps, B, S, seed):
    g = torch.Generator().manual_seed(seed)
    data = torch.randint(0, FIELDS["vocab_size"], (steps, B, S + 1), generator=g)
    return [{"input_ids": d[:, :-1], "labels": d[:, 1:]} for d in data]


def _entry(rank, world, port, fn, args, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        fn(rank, world, *args)
    except Exception:  # report to the parent instead of hanging it
        errq.put((rank, traceback.format_exc()))
        raise


def run_workers(fn, world, args=(), timeout=180):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, f"ranks did not finish within {timeout}s"
    assert not errs, "\n".join(f"rank {r}:\n{e}" for r, e in errs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


# ------------------------------------------------------------------ CPU / gloo
def _collective_worker(rank, world, out_dir):
    import datetime

    from titans_pytorch_b200.parallel.ddp import DataParallelEngine

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False))
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32), device="cpu",
                 engine=DataParallelEngine(reduce="collective"))
    full = _batches(2, 2 * world, 32, seed=1)
    for b in full:
        part = {k: v[rank * 2:(rank + 1) * 2] for k, v in b.items()}
        tr.train_step(part)
    if rank == 0:
        torch.save({k: v.detach().clone() for k, v in model.state_dict().items()}, os.path.join(out_dir, "dp.pt"))
    dist.destroy_process_group()


def test_data_parallel_collective_matches_single_process(tmp_path):
    world = 2
    run_workers(_collective_worker, world, (str(tmp_path),))
    dp = torch.load(tmp_path / "dp.pt")
    # single process: the same per-rank micro-batches, gradients averaged
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False))
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32), device="cpu")
    from titans_pytorch_b200.ops.loss import cross_entropy

    for b in _batches(2, 2 * world, 32, seed=1):
        for r in range(world):
            part = {k: v[r * 2:(r + 1) * 2] for k, v in b.items()}
            logits, _ = model(part["input_ids"])
            (cross_entropy(logits, part["labels"]) / world).backward()
        tr.optimizer_step()
    for k, v in model.state_dict().items():
        torch.testing.assert_close(dp[k], v, atol=1e-5, rtol=1e-4, msg=k)


# ------------------------------------------------------------------ GPUs
def _fused_worker(rank, world, out_dir, steps, graph=False, overlap=True):
    import datetime

    from titans_pytorch_b200.parallel.ddp import DataParallelEngine

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS))
    eng = DataParallelEngine(reduce="fused", overlap=overlap)
    tr = Trainer(model, TrainStepConfig(lr=1e-3, cuda_graph=graph, graph_warmup=2), device=f"cuda:{rank}",
                 engine=eng)
    for b in _batches(steps, 2, 64, seed=1):  # every rank sees the same batch
        tr.train_step({k: v.to(f"cuda:{rank}") for k, v in b.items()})
    torch.cuda.synchronize()
    tr.optimizer.check_errors()
    torch.save({k: v.detach().float().cpu() for k, v in model.state_dict().items()},
               os.path.join(out_dir, f"fused_{rank}.pt"))
    tr._graph = None  # release the captured step before the group goes away
    tr.optimizer.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("overlap", [True, False])
@pytest.mark.parametrize("graph", [False, True])
def test_data_parallel_fused_matches_single_gpu(tmp_path, graph, overlap):
    """2 ranks, fused peer-memory step (eager, or captured in a CUDA graph after two
    eager steps and replayed) against one GPU on the same batches; ``overlap``:
    per-block reduce-scatter on a communication stream during the backward."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    steps = 5 if graph else 3
    run_workers(_fused_worker, 2, (str(tmp_path), steps, graph, overlap), timeout=240)
    f0 = torch.load(tmp_path / "fused_0.pt")
    f1 = torch.load(tmp_path / "fused_1.pt")
    for k in f0:
        assert torch.equal(f0[k], f1[k]), f"ranks hold different weights after the fused step ({k})"
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS))
    tr = Trainer(model, TrainStepConfig(lr=1e-3), device="cuda:0")
    for b in _batches(steps, 2, 64, seed=1):
        tr.train_step(b)
    for k, v in model.state_dict().items():
        torch.testing.assert_close(f0[k], v.float().cpu(), atol=2e-3, rtol=1e-2, msg=k)
