"""Sharded data parallelism: layout arithmetic, gloo ranks on CPU against one
process, and the fused NVLink path on 2 GPUs against one GPU."""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist

import titans_pytorch_b200 as T
from titans_pytorch_b200.parallel.fsdp import ShardLayout, shard_units
from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig

from .test_distributed import FIELDS, _batches, run_workers


def test_layout_partitions_every_group():
    ranges = [(0, 1000 * 8, True), (8000, 333 * 8, False), (10664, 64, False), (10728, 8 * 12345, False)]
    for world in (1, 2, 3, 8):
        lay = ShardLayout(ranges, world)
        for a, n, _ in ranges:
            covered = []
            for r in range(world):
                for fo, so, ln, _ in lay.owned(r):
                    if a <= fo < a + n:
                        assert fo % 8 == 0 and ln % 8 == 0 and so + ln <= lay.n_shard
                        covered.append((fo, ln))
            covered.sort()
            pos = a
            for fo, ln in covered:
                assert fo == pos
                pos += ln
            assert pos == a + n
        # update segments map shard offsets back to the same flat offsets
        active = [(0, 800), (8000, 16), (10728, 8 * 12345)]
        for r in range(world):
            for so, ln, delta, repl in lay.update_segments(active, r):
                fo = so + delta
                assert any(o <= fo and fo + ln <= o + n for o, n in active)


@pytest.mark.parametrize("cls", ["TitansMAG", "TitansMAC"])
def test_units_hold_block_linear_weights(cls):
    model = getattr(T, cls)(T.TitansConfig(**FIELDS, use_kernels=False))
    params, units, unit_params = shard_units(model)
    assert len(units) == FIELDS["num_layers"]
    assert len({id(p) for p in params}) == len(params) == len(list(p for p in model.parameters() if p.requires_grad))
    n_rep = len(params) - sum(len(ps) for ps in unit_params)
    assert all(p.dim() == 2 for ps in unit_params for p in ps)
    assert params[n_rep:] == [p for ps in unit_params for p in ps]


def _fsdp_worker(rank, world, out_dir, cls, reshard=True):
    import datetime

    from titans_pytorch_b200.parallel.fsdp import FullyShardedEngine

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**FIELDS, use_kernels=False))
    eng = FullyShardedEngine(reduce="collective", reshard=reshard)
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32, grad_clip=0.5), device="cpu", engine=eng)
    for b in _batches(3, 2 * world, 32, seed=1):
        r = 0 if cls == "TitansMAC" else rank
        part = {k: v[r * 2:(r + 1) * 2] for k, v in b.items()}
        tr.train_step(part)
    torch.save(tr.optimizer.full_model_state_dict(model), os.path.join(out_dir, f"fsdp_{rank}.pt"))
    tr.optimizer.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("reshard", [True, False])
@pytest.mark.parametrize("cls", ["TitansMAG", "TitansMAL", "TitansMAC", "TitansLMM"])
def test_fsdp_collective_matches_single_process(tmp_path, cls, reshard):
    """FULL_SHARD (``reshard``: units gathered per call into working slots,
    gradients reduce-scattered per call during the backward) and
    SHARD_GRAD_OP against one process.  MAC (reference semantics) writes each
    forward's memory state into the memory weights, so micro-batches run one
    after another on one process differ from micro-batches run side by side;
    its ranks share one batch."""
    world = 2
    run_workers(_fsdp_worker, world, (str(tmp_path), cls, reshard))
    r0 = torch.load(tmp_path / "fsdp_0.pt")
    r1 = torch.load(tmp_path / "fsdp_1.pt")
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**FIELDS, use_kernels=False))
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32, grad_clip=0.5), device="cpu")
    from titans_pytorch_b200.ops.loss import cross_entropy

    for b in _batches(3, 2 * world, 32, seed=1):
        for r in range(world):
            part = {k: v[r * 2:(r + 1) * 2] for k, v in b.items()}
            logits, _ = model(part["input_ids"])
            if cls == "TitansMAC":
                cross_entropy(logits, part["labels"]).backward()
                break
            (cross_entropy(logits, part["labels"]) / world).backward()
        tr.optimizer_step()
    for k, v in model.state_dict().items():
        torch.testing.assert_close(r0[k], v, atol=1e-5, rtol=1e-4, msg=k)
        torch.testing.assert_close(r1[k], v, atol=1e-5, rtol=1e-4, msg=k)


FIELDS4 = dict(FIELDS, num_layers=4)


def _reshard_worker(rank, world, out_dir, cls, accum, ckpt):
    import datetime

    from titans_pytorch_b200.parallel.fsdp import FullyShardedEngine
    from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**FIELDS4, use_kernels=False))
    if ckpt:
        enable_gradient_checkpointing(model)
    eng = FullyShardedEngine(reduce="collective", reshard=True, slots=3)
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32, grad_clip=0.5,
                                        gradient_accumulation_steps=accum), device="cpu", engine=eng)
    assert tr.optimizer.R == 3 and tr.optimizer.reshard
    for b in _batches(2 * accum, 2 * world, 64, seed=2):
        r = 0 if cls == "TitansMAC" else rank
        tr.train_step({k: v[r * 2:(r + 1) * 2] for k, v in b.items()})
    torch.save(tr.optimizer.full_model_state_dict(model), os.path.join(out_dir, f"rs_{rank}.pt"))
    tr.optimizer.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("cls,accum,ckpt", [("TitansMAG", 1, False), ("TitansMAG", 2, False),
                                            ("TitansMAC", 1, False), ("TitansMAC", 2, False),
                                            ("TitansMAL", 1, True)])
def test_fsdp_reshard_slot_reuse_matches_single_process(tmp_path, cls, accum, ckpt):
    """4 blocks over 3 working slots (slots reused within a forward and a
    backward), MAC's 2 segments (every block called twice, its gradients
    reduce-scattered per call and accumulated), gradient accumulation over
    micro-batches, and MAL with activation checkpointing (recompute inside the
    backward), against one process."""
    world = 2
    run_workers(_reshard_worker, world, (str(tmp_path), cls, accum, ckpt))
    r0 = torch.load(tmp_path / "rs_0.pt")
    r1 = torch.load(tmp_path / "rs_1.pt")
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**FIELDS4, use_kernels=False))
    if ckpt:
        from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

        enable_gradient_checkpointing(model)
    tr = Trainer(model, TrainStepConfig(lr=1e-3, dtype=torch.float32, grad_clip=0.5), device="cpu")
    from titans_pytorch_b200.ops.loss import cross_entropy

    batches = _batches(2 * accum, 2 * world, 64, seed=2)
    for i in range(0, len(batches), accum):
        for b in batches[i:i + accum]:
            for r in range(world):
                part = {k: v[r * 2:(r + 1) * 2] for k, v in b.items()}
                logits, _ = model(part["input_ids"])
                if cls == "TitansMAC":
                    (cross_entropy(logits, part["labels"]) / accum).backward()
                    break
                (cross_entropy(logits, part["labels"]) / (world * accum)).backward()
        tr.optimizer_step()
    for k, v in model.state_dict().items():
        torch.testing.assert_close(r0[k], v, atol=1e-5, rtol=1e-4, msg=k)
        torch.testing.assert_close(r1[k], v, atol=1e-5, rtol=1e-4, msg=k)


# ------------------------------------------------------------------ GPUs
def _fused_worker(rank, world, out_dir, steps, graph, reshard=True):
    import datetime

    from titans_pytorch_b200.ops._ext import ext
    from titans_pytorch_b200.parallel.fsdp import FullyShardedEngine

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS4))
    eng = FullyShardedEngine(reduce="fused", reshard=reshard)
    tr = Trainer(model, TrainStepConfig(lr=1e-3, cuda_graph=graph, graph_warmup=2), device=f"cuda:{rank}",
                 engine=eng)
    for b in _batches(steps, 2, 64, seed=1):  # every rank sees the same batch
        tr.train_step({k: v.to(f"cuda:{rank}") for k, v in b.items()})
    torch.cuda.synchronize()
    tr.optimizer.check_errors()
    assert int(ext().kernel_error_status(rank, True)) == 0
    sd = tr.optimizer.full_model_state_dict(model)
    torch.cuda.synchronize()
    torch.save({k: v.float() for k, v in sd.items()}, os.path.join(out_dir, f"fused_{rank}.pt"))
    tr._graph = None  # release the captured step before the group goes away
    dist.barrier()
    tr.optimizer.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("reshard", [True, False])
@pytest.mark.parametrize("graph", [False, True])
def test_fsdp_fused_matches_single_gpu(tmp_path, graph, reshard):
    """2 ranks, sharded parameters with the fused gather-GEMM prefetch (eager, or
    captured in a CUDA graph after two eager steps and replayed) against one GPU;
    ``reshard``: FULL_SHARD (working slots, re-gathers and per-call reductions
    on side streams during the backward)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    steps = 5 if graph else 3
    run_workers(_fused_worker, 2, (str(tmp_path), steps, graph, reshard), timeout=240)
    f0 = torch.load(tmp_path / "fused_0.pt")
    f1 = torch.load(tmp_path / "fused_1.pt")
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS4))
    tr = Trainer(model, TrainStepConfig(lr=1e-3), device="cuda:0")
    for b in _batches(steps, 2, 64, seed=1):
        tr.train_step(b)
    for k, v in model.state_dict().items():
        assert torch.equal(f0[k], f1[k]), f"ranks differ on {k}"
        torch.testing.assert_close(f0[k], v.float().cpu(), atol=2e-3, rtol=1e-2, msg=k)
