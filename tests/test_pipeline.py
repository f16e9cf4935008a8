"""MAC pipeline parallelism (layers split into stages, segments as micro-batches):
gloo ranks against one process over the whole model."""

from __future__ import annotations

import datetime
import os

import pytest
import torch
import torch.distributed as dist

import titans_pytorch_b200 as T
from titans_pytorch_b200.ops.loss import cross_entropy
from titans_pytorch_b200.parallel.pipeline import MACPipeline, split_layers
from tests.test_distributed import run_workers

FIELDS = dict(dim=64, num_heads=4, num_layers=4, vocab_size=97, window_size=8, chunk_size=8,
              num_persistent_tokens=4, dropout=0.0, max_seq_len=256, ffn_mult=2.0, num_memory_layers=2,
              memory_hidden_mult=2.0, init_std=0.2)


def _batch(B, S, seed):
    g = torch.Generator().manual_seed(seed)
    d = torch.randint(0, FIELDS["vocab_size"], (B, S + 1), generator=g)
    lab = d[:, 1:].clone()
    lab[0, 3] = -100  # an ignored position
    return d[:, :-1], lab


def _pp_worker(rank, world, out_dir):
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    names = {p: n for n, p in model.named_parameters()}
    pipe = MACPipeline(model)
    ids, lab = _batch(2, 28, seed=4)  # 3 full segments of 8 and one of 4
    loss, states = pipe.forward_backward(ids, lab)
    grads = {names[p]: p.grad.clone() for p in pipe.parameters() if p.grad is not None}
    norm = pipe.clip_grad_norm_(1e9)
    with torch.no_grad():
        loss2, _ = pipe.forward_backward(ids, lab, states)
    torch.save({"loss": loss, "loss2": loss2, "grads": grads, "norm": norm, "lo": pipe.lo, "hi": pipe.hi,
                "states": [(s.weights, s.momentum) for s in states]}, os.path.join(out_dir, f"pp{rank}.pt"))
    dist.destroy_process_group()


def test_split_layers():
    assert split_layers(4, 2) == [(0, 2), (2, 4)]
    assert split_layers(5, 3) == [(0, 2), (2, 4), (4, 5)]
    with pytest.raises(ValueError):
        split_layers(2, 3)


@pytest.mark.parametrize("world", [2, 3])
def test_mac_pipeline_matches_one_process(tmp_path, world):
    run_workers(_pp_worker, world, (str(tmp_path),))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    ids, lab = _batch(2, 28, seed=4)
    logits, states = model(ids)
    loss = cross_entropy(logits, lab)
    loss.backward()
    ref = {n: p.grad for n, p in model.named_parameters() if p.grad is not None}
    norm = torch.sqrt(sum(g.float().pow(2).sum() for g in ref.values()))
    with torch.no_grad():
        logits2, _ = model(ids, [s.clone() for s in states])
        loss2 = cross_entropy(logits2, lab)
    seen = set()
    for r in range(world):
        pp = torch.load(tmp_path / f"pp{r}.pt")
        torch.testing.assert_close(pp["loss"], loss.detach(), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(pp["loss2"], loss2, atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(pp["norm"], norm, atol=1e-5, rtol=1e-4)
        for n, g in pp["grads"].items():
            torch.testing.assert_close(g, ref[n], atol=2e-6, rtol=1e-4, msg=n)
            seen.add(n)
        for (w, m), s in zip(pp["states"], states[pp["lo"]:pp["hi"]], strict=True):
            torch.testing.assert_close(w, s.weights, atol=1e-6, rtol=1e-5)
            torch.testing.assert_close(m, s.momentum, atol=1e-6, rtol=1e-5)
    assert seen == set(ref), set(ref) ^ seen  # every parameter's gradient lives on some stage


def test_mac_pipeline_one_rank_and_rejects_other_models():
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    pipe = MACPipeline(model)
    assert (pipe.lo, pipe.hi, pipe.first, pipe.last) == (0, 4, True, True)
    ids, lab = _batch(2, 16, seed=1)
    loss, _ = pipe.forward_backward(ids, lab)
    g = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    torch.manual_seed(0)
    ref = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    l2 = cross_entropy(ref(ids)[0], lab)
    l2.backward()
    torch.testing.assert_close(loss, l2.detach(), atol=1e-5, rtol=1e-5)
    for n, p in ref.named_parameters():
        if p.grad is not None:
            torch.testing.assert_close(g[n], p.grad, atol=2e-6, rtol=1e-4, msg=n)
    with pytest.raises(NotImplementedError):
        MACPipeline(T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False)))


def _pp_train_worker(rank, world, out_dir):
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    names = {p: n for n, p in model.named_parameters()}
    pipe = MACPipeline(model)
    opt = pipe.make_optimizer(lr=1e-3)
    losses = []
    for seed in range(3):
        ids, lab = _batch(2, 24, seed=seed)
        losses.append(float(pipe.train_step({"input_ids": ids, "labels": lab}, opt, max_grad_norm=0.5)))
    own = {names[p]: p.detach().clone() for p in pipe.parameters()}
    torch.save({"losses": losses, "params": own}, os.path.join(out_dir, f"tr{rank}.pt"))
    dist.destroy_process_group()


def test_mac_pipeline_training_matches_one_process(tmp_path):
    """Three AdamW steps with a global-norm clip: every stage's parameters equal the
    one-process run's (the clip norm is reduced over the stages)."""
    from titans_pytorch_b200.train.optim import FusedAdamW

    run_workers(_pp_train_worker, 2, (str(tmp_path),))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    opt = FusedAdamW(model.parameters(), lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=0.5,
                     use_kernels=False)
    losses = []
    for seed in range(3):
        ids, lab = _batch(2, 24, seed=seed)
        loss = cross_entropy(model(ids)[0], lab)
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(float(loss.detach()))
    ref = dict(model.named_parameters())
    for r in range(2):
        tr = torch.load(tmp_path / f"tr{r}.pt")
        assert tr["losses"] == pytest.approx(losses, rel=1e-5, abs=1e-5)
        for n, p in tr["params"].items():
            # AdamW divides by the root of the second moment, so an fp32 rounding
            # difference in a gradient near zero can move a weight by a small fraction
            # of the step size (1e-3); a missing clip or tied-weight sum moves far more.
            torch.testing.assert_close(p, ref[n].detach(), atol=2e-4, rtol=0, msg=n)


def _gpu_pp_worker(rank, world, out_dir):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        fields = {**FIELDS, "dim": 256, "num_heads": 4, "chunk_size": 128, "window_size": 128, "vocab_size": 512,
                  "init_std": 0.05}
        g = torch.Generator().manual_seed(7)
        d = torch.randint(0, 512, (2, 513), generator=g)
        ids, lab = d[:, :-1].cuda(), d[:, 1:].cuda()
        torch.manual_seed(0)
        ref = T.TitansMAC(T.TitansConfig(**fields)).cuda().to(torch.bfloat16)
        torch.manual_seed(0)
        model = T.TitansMAC(T.TitansConfig(**fields)).cuda().to(torch.bfloat16)
        loss_ref = cross_entropy(ref(ids)[0], lab)
        loss_ref.backward()
        pipe = MACPipeline(model)
        loss, _ = pipe.forward_backward(ids, lab)
        rg = dict(ref.named_parameters())
        names = {p: n for n, p in model.named_parameters()}
        worst = 0.0
        for p in pipe.parameters():
            a, b = p.grad.float(), rg[names[p]].grad.float()
            worst = max(worst, ((a - b).norm() / b.norm().clamp_min(1e-12)).item())
        torch.save({"loss": float(loss), "loss_ref": float(loss_ref), "worst": worst},
                   os.path.join(out_dir, f"g{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gpu_mac_pipeline_two_ranks(tmp_path):
    """Two NCCL stages on bf16 kernels against the one-GPU model: the loss and each
    stage's gradients (relative norm error of bf16 rounding)."""
    run_workers(_gpu_pp_worker, 2, (str(tmp_path),), timeout=300)
    for r in range(2):
        res = torch.load(tmp_path / f"g{r}.pt")
        assert abs(res["loss"] - res["loss_ref"]) < 2e-2 * abs(res["loss_ref"]), res
        assert res["worst"] < 0.05, res


def _pp_engine_worker(rank, world, out_dir):
    from titans_pytorch_b200.parallel.pipeline import PipelineEngine
    from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    names = {p: n for n, p in model.named_parameters()}
    cfg = TrainStepConfig(lr=1e-3, dtype=torch.float32, gradient_accumulation_steps=2, grad_clip=0.5)
    tr = Trainer(model, cfg, device="cpu", engine=PipelineEngine())
    for seed in range(4):  # two optimizer steps of two micro-batches
        ids, lab = _batch(2, 24, seed=seed)
        tr.train_step({"input_ids": ids, "labels": lab})
    own = {names[p]: p.detach().clone() for p in tr.engine.pipe.parameters()}
    torch.save(own, os.path.join(out_dir, f"en{rank}.pt"))
    dist.destroy_process_group()


def test_pipeline_engine_gradient_accumulation(tmp_path):
    """The Trainer with PipelineEngine and two accumulated micro-batches per step equals
    the one-process Trainer (the tied weight's gradient is summed once per step)."""
    from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig

    run_workers(_pp_engine_worker, 2, (str(tmp_path),))
    torch.manual_seed(0)
    model = T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False))
    cfg = TrainStepConfig(lr=1e-3, dtype=torch.float32, gradient_accumulation_steps=2, grad_clip=0.5)
    tr = Trainer(model, cfg, device="cpu")
    for seed in range(4):
        ids, lab = _batch(2, 24, seed=seed)
        tr.train_step({"input_ids": ids, "labels": lab})
    ref = dict(model.named_parameters())
    for r in range(2):
        for n, p in torch.load(tmp_path / f"en{r}.pt").items():
            torch.testing.assert_close(p, ref[n].detach(), atol=2e-4, rtol=0, msg=n)
