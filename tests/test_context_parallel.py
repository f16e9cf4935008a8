"""Context parallelism (a sequence split over ranks): equal to the unsharded model.

CPU: gloo ranks against one process over the whole sequence (logits, memory
states, the carried-state second call and the averaged parameter gradients).
GPU: the RoPE position offset of the attention kernel, and two NCCL ranks
against the unsharded model on bf16 kernels.
"""

from __future__ import annotations

import datetime
import os

import pytest
import torch
import torch.distributed as dist

import titans_pytorch_b200 as T
from titans_pytorch_b200.ops.attention import window_attention, window_attention_reference
from titans_pytorch_b200.ops.loss import cross_entropy
from titans_pytorch_b200.parallel.context import (ContextShard, enable_context_parallel, shard_batch,
                                                  shard_sequence)
from tests.test_distributed import run_workers

FIELDS = dict(dim=64, num_heads=4, num_layers=2, vocab_size=97, window_size=8, chunk_size=32,
              num_persistent_tokens=4, dropout=0.0, max_seq_len=256, ffn_mult=2.0, num_memory_layers=2,
              memory_hidden_mult=2.0, init_std=0.2)


def _batch(B, S, seed, vocab=97):
    g = torch.Generator().manual_seed(seed)
    d = torch.randint(0, vocab, (B, S + 1), generator=g)
    return {"input_ids": d[:, :-1], "labels": d[:, 1:]}


def _run(model, batch, reduce_grads=None):
    logits, states = model(batch["input_ids"])
    cross_entropy(logits, batch["labels"]).backward()
    grads = {}
    for n, p in model.named_parameters():
        if p.grad is not None:
            g = p.grad.detach().clone()
            if reduce_grads is not None:
                reduce_grads(g)
            grads[n] = g
    with torch.no_grad():
        logits2, states2 = model(batch["input_ids"], [s.clone() for s in states])
    return logits.detach(), states, grads, logits2, states2


def _cp_worker(rank, world, out_dir, cls, fields, S, ckpt=False):
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**fields, use_kernels=False))
    shard = enable_context_parallel(model)
    if ckpt:  # the memory update then runs outside the recomputed region, with its own halo
        from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

        enable_gradient_checkpointing(model)
    assert (shard.rank, shard.world) == (rank, world)
    part = shard_batch(_batch(2, S, seed=3), shard)

    def avg(g):
        dist.all_reduce(g)
        g.div_(world)

    logits, states, grads, logits2, states2 = _run(model, part, avg)

    def gather(t):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts, dim=1)

    out = {"logits": gather(logits), "logits2": gather(logits2), "grads": grads,
           "states": [(s.weights, s.momentum) for s in states],
           "states2": [(s.weights, s.momentum) for s in states2]}
    torch.save(out, os.path.join(out_dir, f"cp{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("cls,world,S,ckpt", [("TitansMAG", 2, 32, False), ("TitansMAL", 2, 32, False),
                                              ("TitansLMM", 2, 32, False), ("TitansMAG", 4, 32, False),
                                              ("TitansMAG", 2, 32, True), ("TitansMAL", 2, 32, True)])
def test_context_parallel_matches_whole_sequence(tmp_path, cls, world, S, ckpt):
    run_workers(_cp_worker, world, (str(tmp_path), cls, FIELDS, S, ckpt))
    torch.manual_seed(0)
    model = getattr(T, cls)(T.TitansConfig(**FIELDS, use_kernels=False))
    logits, states, grads, logits2, states2 = _run(model, _batch(2, S, seed=3))
    for r in range(world):
        cp = torch.load(tmp_path / f"cp{r}.pt")
        torch.testing.assert_close(cp["logits"], logits, atol=2e-5, rtol=1e-4)
        torch.testing.assert_close(cp["logits2"], logits2, atol=2e-5, rtol=1e-4)
        for (w, m), s in zip(cp["states"], states, strict=True):
            torch.testing.assert_close(w, s.weights, atol=1e-6, rtol=1e-4)
            torch.testing.assert_close(m, s.momentum, atol=1e-6, rtol=1e-4)
        for (w, m), s in zip(cp["states2"], states2, strict=True):
            torch.testing.assert_close(w, s.weights, atol=1e-6, rtol=1e-4)
        assert cp["grads"].keys() == grads.keys()
        for n, g in grads.items():
            torch.testing.assert_close(cp["grads"][n], g, atol=2e-6, rtol=1e-3, msg=n)


def test_attention_position_offset_reference():
    """A shard with its halo and the global offset reproduces the whole sequence's rows."""
    torch.manual_seed(0)
    B, S, H, d, P, w = 2, 48, 2, 16, 3, 8
    qkv = torch.randn(B, S, 3 * H * d)
    pkv = torch.randn(1, P, 2 * H * d)
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d))
    full = window_attention_reference(qkv, pkv, H, w, d ** -0.5, inv)
    for s0, T_ in ((16, 16), (32, 16), (0, 16)):
        h = min(w - 1, s0)
        part = window_attention_reference(qkv[:, s0 - h:s0 + T_], pkv, H, w, d ** -0.5, inv, pos_offset=s0 - h)
        torch.testing.assert_close(part[:, h:], full[:, s0:s0 + T_], atol=1e-5, rtol=1e-5)


def test_context_parallel_rejects_mac_and_paper():
    with pytest.raises(NotImplementedError):
        enable_context_parallel(T.TitansMAC(T.TitansConfig(**FIELDS, use_kernels=False)))
    with pytest.raises(NotImplementedError):
        enable_context_parallel(T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False, semantics="paper")))


def test_shard_sequence_split():
    t = torch.arange(2 * 12).view(2, 12)
    parts = [shard_sequence(t, ContextShard(None, r, 3)) for r in range(3)]
    assert torch.equal(torch.cat(parts, dim=1), t)
    with pytest.raises(ValueError):
        shard_sequence(t, ContextShard(None, 0, 5))


# ------------------------------------------------------------------ GPUs
@pytest.mark.gpu
@pytest.mark.parametrize("hd", [64, 96])
def test_gpu_attention_position_offset(hd):
    """The kernel's main-row RoPE offset against the fp32 reference, forward and backward."""
    torch.manual_seed(0)
    B, T_, H, P, w, off = 2, 512, 4, 4, 128, 1000
    dev = "cuda"
    qkv = torch.randn(B, T_, 3 * H * hd, device=dev, dtype=torch.bfloat16, requires_grad=True)
    pkv = torch.randn(1, P, 2 * H * hd, device=dev, dtype=torch.bfloat16, requires_grad=True)
    inv = 1.0 / (10000 ** (torch.arange(0, hd, 2, device=dev).float() / hd))
    do = torch.randn(B, T_, H, hd, device=dev, dtype=torch.bfloat16)
    o = window_attention(qkv, pkv, H, window=w, inv_freq=inv, use_kernels=True, pos_offset=off)
    o.backward(do)
    q32 = qkv.detach().float().requires_grad_(True)
    p32 = pkv.detach().float().requires_grad_(True)
    r = window_attention_reference(q32, p32, H, w, hd ** -0.5, inv, pos_offset=off)
    r.backward(do.float())
    torch.testing.assert_close(o.float(), r, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(qkv.grad.float(), q32.grad, atol=6e-2, rtol=5e-2)
    torch.testing.assert_close(pkv.grad.float(), p32.grad, atol=2e-1, rtol=5e-2)
    # offset 0 differs: the offset really reaches the rotation
    o0 = window_attention(qkv.detach(), pkv.detach(), H, window=w, inv_freq=inv, use_kernels=True)
    assert (o0.float() - o.detach().float()).abs().max() > 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("layers", [1, 2, 3])
def test_gpu_sharded_memory_step_one_rank(layers):
    """On one shard the sharded update (tcgen05 gradients in fp32, then the
    update kernel) equals the fused update."""
    from titans_pytorch_b200.ops.memory import memory_step, memory_step_sharded

    torch.manual_seed(0)
    B, T_, D, Hd = 2, 1024, 256, 512
    dev, bf = "cuda", torch.bfloat16
    k = torch.nn.functional.normalize(torch.randn(B, T_, D, device=dev), dim=-1).to(bf)
    v = torch.randn(B, T_, D, device=dev, dtype=bf)
    x = torch.randn(B, T_, D, device=dev, dtype=bf)
    dims = [D, D] if layers == 1 else [D] + [Hd] * (layers - 1) + [D]
    ws = [(torch.randn(dims[i + 1], dims[i], device=dev) * 0.05).to(bf) for i in range(layers)]
    ms = [(torch.randn_like(w.float()) * 0.01).to(bf) for w in ws]
    gw = [(torch.randn(D, D, device=dev) * 0.02).to(bf) for _ in range(3)]
    gb = [torch.zeros(D, device=dev, dtype=bf) for _ in range(3)]
    lin = layers == 1
    w1, m1 = memory_step(k, v, x, ws, ms, gw, gb, 0.1, 0.9, "silu", lin)
    w2, m2 = memory_step_sharded(k, v, x, ws, ms, gw, gb, 0.1, 0.9, "silu", lin, None, ContextShard())
    for a, b in zip(w1 + m1, w2 + m2, strict=True):
        torch.testing.assert_close(b.float(), a.float(), atol=2e-3, rtol=2e-2)


def _gpu_cp_worker(rank, world, out_dir, cls, S):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        fields = {**FIELDS, "dim": 256, "num_heads": 4, "window_size": 128, "vocab_size": 512, "max_seq_len": S,
                  "init_std": 0.05}
        batch = {k: v.cuda() for k, v in _batch(2, S, seed=5, vocab=512).items()}
        torch.manual_seed(0)
        ref = getattr(T, cls)(T.TitansConfig(**fields)).cuda().to(torch.bfloat16)
        torch.manual_seed(0)
        model = getattr(T, cls)(T.TitansConfig(**fields)).cuda().to(torch.bfloat16)
        with torch.no_grad():
            full, fstates = ref(batch["input_ids"])
            shard = enable_context_parallel(model)
            part, states = model(shard_batch(batch, shard)["input_ids"])
        mine = shard_sequence(full, shard)
        err = (part.float() - mine.float()).abs().max().item()
        scale = mine.float().abs().max().item()
        serr = max((a.float() - b.float()).abs().max().item() / (b.float().abs().max().item() + 1e-12)
                   for s, f in zip(states, fstates, strict=True) for a, b in zip(s.weights, f.weights, strict=True))
        torch.save({"err": err, "scale": scale, "state_err": serr}, os.path.join(out_dir, f"g{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("cls", ["TitansMAG", "TitansMAL"])
def test_gpu_context_parallel_two_ranks(tmp_path, cls):
    run_workers(_gpu_cp_worker, 2, (str(tmp_path), cls, 1024), timeout=300)
    for r in range(2):
        res = torch.load(tmp_path / f"g{r}.pt")
        assert res["err"] <= 0.05 * res["scale"] + 0.05, res
        assert res["state_err"] < 0.02, res


def _cp_dp_worker(rank, world, out_dir, S):
    """Four ranks: context-parallel pairs {0, 1} and {2, 3}, each pair on its own sequence."""
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    torch.manual_seed(0)
    model = T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False))
    shard = enable_context_parallel(model, groups[rank // 2])
    assert (shard.rank, shard.world) == (rank % 2, 2)
    ids, lab = (t[rank // 2:rank // 2 + 1] for t in (_batch(2, S, seed=9)["input_ids"],
                                                    _batch(2, S, seed=9)["labels"]))
    part = shard_batch({"input_ids": ids, "labels": lab}, shard)
    logits, _ = model(part["input_ids"])
    cross_entropy(logits, part["labels"]).backward()
    grads = {}
    for n, p in model.named_parameters():
        if p.grad is not None:
            g = p.grad.detach().clone()
            dist.all_reduce(g)  # the data-parallel average over all four ranks
            grads[n] = g / world
    torch.save(grads, os.path.join(out_dir, f"cpdp{rank}.pt"))
    dist.destroy_process_group()


def test_context_parallel_inside_data_parallel(tmp_path):
    """Two data-parallel replicas, each a context-parallel pair: the gradients averaged
    over all ranks equal the mean of the two sequences' whole-sequence gradients."""
    S = 32
    run_workers(_cp_dp_worker, 4, (str(tmp_path), S))
    b = _batch(2, S, seed=9)
    ref = {}
    for i in range(2):
        torch.manual_seed(0)
        model = T.TitansMAG(T.TitansConfig(**FIELDS, use_kernels=False))
        logits, _ = model(b["input_ids"][i:i + 1])
        cross_entropy(logits, b["labels"][i:i + 1]).backward()
        for n, p in model.named_parameters():
            if p.grad is not None:
                ref[n] = ref.get(n, 0) + p.grad / 2
    for r in range(4):
        got = torch.load(tmp_path / f"cpdp{r}.pt")
        assert got.keys() == ref.keys()
        for n, g in ref.items():
            torch.testing.assert_close(got[n], g, atol=2e-6, rtol=1e-3, msg=n)
