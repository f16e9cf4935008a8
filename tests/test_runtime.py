"""Checkpoint/hub formats, generation, datasets and CLIs (CPU)."""

from __future__ import annotations

import json
import os

import pytest
import torch
import torch.nn.functional as F

import titans_pytorch_b200 as T
from tests.conftest import import_reference
from titans_pytorch_b200.inference import generate as G
from titans_pytorch_b200.utils import checkpoint as C
from titans_pytorch_b200.utils import hub as H

FIELDS = dict(dim=32, num_heads=2, num_layers=2, vocab_size=64, window_size=8, chunk_size=16,
              num_persistent_tokens=2, dropout=0.0, max_seq_len=128, ffn_mult=2.0, memory_hidden_mult=2.0)


def tiny(kind="mag"):
    torch.manual_seed(0)
    return T.create_model(kind, T.TitansConfig(**FIELDS))


@pytest.mark.parametrize("kind", ["mac", "mag", "mal", "lmm"])
def test_checkpoint_loads_in_reference_loader(tmp_path, kind):
    ref = import_reference()
    m = tiny(kind)
    path = C.save_checkpoint(str(tmp_path / "c.pt"), m, global_step=7)
    ck = torch.load(path, weights_only=False)
    cls = {"mac": ref.TitansMAC, "mag": ref.TitansMAG, "mal": ref.TitansMAL, "lmm": ref.TitansLMM}[ck["model_type"]]
    rm = cls(ref.TitansConfig(**ck["config"]))          # the reference's loader steps
    rm.load_state_dict(ck["model_state_dict"])
    ids = torch.randint(0, 64, (1, 20))
    with torch.no_grad():
        torch.testing.assert_close(rm(ids)[0], m(ids)[0], atol=1e-5, rtol=1e-4)


def test_load_reference_trainer_checkpoint(tmp_path):
    """A reference pretrain.py checkpoint: config = trainer flags, no model_type, compiled-key prefix."""
    ref = import_reference()
    rm = ref.TitansMAL(ref.TitansConfig(**FIELDS))
    sd = {"_orig_mod." + k: v for k, v in rm.state_dict().items()}
    torch.save({"model_state_dict": sd, "config": {**FIELDS, "lr": 1e-3, "batch_size": 4, "model": "mal"},
                "global_step": 3}, tmp_path / "ref.pt")
    m, ck = C.load_model(str(tmp_path / "ref.pt"))
    assert isinstance(m, T.TitansMAL) and ck["global_step"] == 3


def test_resume_restores_optimizer_and_rng(tmp_path):
    from titans_pytorch_b200.train.trainer import Trainer, TrainStepConfig

    m = tiny()
    tr = Trainer(m, TrainStepConfig(lr=1e-3, dtype=torch.float32), device="cpu")
    ids = torch.randint(0, 64, (2, 33))
    b = {"input_ids": ids[:, :-1], "labels": ids[:, 1:]}
    tr.train_step(b)
    C.save_checkpoint(str(tmp_path / "r.pt"), tr.model, tr.optimizer, global_step=tr.global_step)
    after = float(tr.train_step(b))
    m2 = tiny()
    tr2 = Trainer(m2, TrainStepConfig(lr=1e-3, dtype=torch.float32), device="cpu")
    C.load_checkpoint(str(tmp_path / "r.pt"), tr2.model, tr2.optimizer)
    assert abs(float(tr2.train_step(b)) - after) < 1e-6


def test_hub_roundtrip(tmp_path):
    m = tiny("mac")
    d = H.push_to_hub(m, "user/titans-test", local_dir=str(tmp_path / "hub"), tokenizer_name=None)
    meta = json.load(open(os.path.join(d, "config.json")))
    assert meta["model_type"] == "mac" and "dim" in meta["titans_config"]
    m2 = H.load_from_hub(d)
    for (k, v), (k2, v2) in zip(m.state_dict().items(), m2.state_dict().items()):
        assert k == k2 and torch.equal(v, v2)
    assert H._estimate_params(meta["titans_config"], "mac") == sum(p.numel() for p in m.parameters())


def _ref_filters(logits, generated, penalty, top_k, top_p):
    """The reference's per-token loops (scripts/inference.py:367-397), for comparison."""
    logits = logits.clone()
    for i in range(generated.shape[0]):
        for t in set(generated[i].tolist()):
            logits[i, t] /= penalty
    kth = torch.topk(logits, top_k)[0][..., -1, None]
    logits[logits < kth] = float("-inf")
    s, idx = torch.sort(logits, descending=True)
    cum = torch.cumsum(F.softmax(s, dim=-1), dim=-1)
    rem = cum > top_p
    rem[..., 1:] = rem[..., :-1].clone()
    rem[..., 0] = False
    logits[rem.scatter(1, idx, rem)] = float("-inf")
    return logits


def test_sampling_filters_match_reference_loops():
    torch.manual_seed(0)
    logits = torch.randn(3, 50)
    gen = torch.randint(0, 50, (3, 12))
    ours = G.top_p_filter(G.top_k_filter(G.apply_repetition_penalty(logits, gen, 1.3), 10), 0.8)
    torch.testing.assert_close(ours, _ref_filters(logits, gen, 1.3, 10, 0.8))


def test_generate_greedy_stream_and_eos():
    m = tiny().eval()
    ids = torch.randint(0, 64, (2, 5))
    out, st = G.generate(m, ids, 6, greedy=True)
    assert out.shape == (2, 11) and len(st) == 2
    again, _ = G.generate(tiny().eval(), ids, 6, greedy=True)
    assert torch.equal(out, again)
    chunks = list(G.generate(m, ids, 4, greedy=True, stream=True))
    assert len(chunks) == 4 and chunks[-1][0].shape[1] == 9
    first, _ = G.generate(tiny().eval(), ids[:1], 1, greedy=True)
    eos = int(first[0, -1])
    stopped, _ = G.generate(tiny().eval(), ids[:1], 10, greedy=True, eos_token_id=eos)
    assert stopped.shape[1] == 6


def test_continuous_batcher_and_static_cache():
    m = tiny().eval()
    cb = G.ContinuousBatcher(m, max_batch_size=2, context=16)
    rids = [cb.add_request(torch.randint(0, 64, (n,)), max_new_tokens=k) for n, k in ((5, 3), (7, 2), (4, 4))]
    done = cb.run()
    assert sorted(d["id"] for d in done) == sorted(rids)
    cache = G.StaticKVCache(G.KVCacheConfig(max_batch_size=2, max_seq_len=8, num_layers=1, num_heads=1,
                                            head_dim=4, dtype=torch.float32))
    k = torch.randn(2, 1, 3, 4)
    kk, vv = cache.update(0, k, k, torch.tensor([0, 1]))
    assert kk.shape == (2, 1, 3, 4)


def test_prefill_equals_chunked_calls():
    m = tiny("mag").eval()
    ids = torch.randint(0, 64, (1, 40))
    last, st = G.prefill(m, ids, chunk=16)
    s = None
    for a in range(0, 40, 16):
        lg, s = m(ids[:, a:a + 16], states=s)
    torch.testing.assert_close(last, lg[:, -1])


def test_datasets(tmp_path):
    from titans_pytorch_b200.utils import data as D

    ds = D.SyntheticDataset(64, 16, 10, seed=1)
    it = ds[3]
    assert it["input_ids"].shape == (16,) and torch.equal(it["input_ids"][1:], it["labels"][:-1])
    p = tmp_path / "t.txt"
    p.write_text("hello world " * 20)
    cd = D.CharLevelDataset(str(p), 64, 8)
    assert len(cd) == len("hello world " * 20) - 8


def test_cli_pretrain_infer_eval_pretokenize(tmp_path, capsys):
    from titans_pytorch_b200.cli import eval_perplexity, inference, pretokenize, pretrain

    text = tmp_path / "corpus.txt"
    text.write_text("the quick brown fox jumps over the lazy dog. " * 40)
    ck = tmp_path / "ck"
    common = ["--model", "mag", "--dim", "32", "--num-heads", "2", "--num-layers", "1", "--vocab-size", "128",
              "--window-size", "8", "--chunk-size", "16", "--num-persistent-tokens", "2", "--seq-len", "32",
              "--batch-size", "2", "--mixed-precision", "none", "--num-workers", "0", "--log-every", "1",
              "--checkpoint-dir", str(ck), "--save-every", "0"]
    pretrain.main(common + ["--data", str(text), "--max-steps", "3"])
    final = ck / "final_model.pt"
    assert final.exists()
    inference.main(["--checkpoint", str(final), "--prompt", "the", "--max-tokens", "5", "--device", "cpu"])
    inference.main(["--checkpoint", str(final), "--prompt", "the", "--max-tokens", "5", "--device", "cpu",
                    "--decoder", "incremental", "--quantize", "int8"])
    eval_perplexity.main(["--checkpoint", str(final), "--data", str(text), "--max-length", "64", "--stride",
                          "32", "--device", "cpu", "--max-tokens", "300"])
    eval_perplexity.main(["--checkpoint", str(final), "--data", str(text), "--use-memory", "--chunk-size", "32",
                          "--device", "cpu", "--max-tokens", "300"])
    out = capsys.readouterr().out
    assert "perplexity" in out
    pytest.importorskip("datasets")
    pretokenize.main(["--input", str(text), "--output", str(tmp_path / "tok"), "--seq-len", "32",
                      "--vocab-size", "128"])
    pretrain.main(common + ["--local-dataset", str(tmp_path / "tok"), "--max-steps", "2"])


@pytest.mark.parametrize("kind", ["mac", "mag"])
def test_weight_cache_does_not_outlive_a_forward(kind):
    """Derived weights cached within one forward must reflect in-place weight updates."""
    m = tiny(kind).eval()
    ids = torch.randint(0, 64, (1, 40))
    with torch.no_grad():
        a, _ = m(ids)
        for p in m.parameters():
            p.mul_(1.5)
        b, _ = m(ids)
    fresh = tiny(kind).eval()
    fresh.load_state_dict(m.state_dict())
    with torch.no_grad():
        c, _ = fresh(ids)
    assert not torch.allclose(a, b)
    torch.testing.assert_close(b, c)


@pytest.mark.parametrize("kind", ["mal", "mag", "lmm"])
def test_gradient_checkpointing_runs_update_once_and_matches(kind):
    """Checkpointed blocks (memory update outside the recomputed region) equal plain blocks."""
    import copy

    from titans_pytorch_b200.ops.loss import cross_entropy
    from titans_pytorch_b200.utils.perf import enable_gradient_checkpointing

    a = tiny(kind)
    b = copy.deepcopy(a)
    enable_gradient_checkpointing(b)
    calls = {"n": 0}
    for blk in b.blocks:
        orig = blk.memory._update

        def counted(*args, _orig=orig, **kw):
            calls["n"] += 1
            return _orig(*args, **kw)

        blk.memory._update = counted
    ids = torch.randint(0, 64, (2, 33))
    la, sa = a(ids[:, :-1])
    lb, sb = b(ids[:, :-1])
    cross_entropy(la, ids[:, 1:]).backward()
    cross_entropy(lb, ids[:, 1:]).backward()
    assert calls["n"] == len(b.blocks)  # once per block, not again in the recompute
    torch.testing.assert_close(la, lb)
    for pa, pb in zip(a.parameters(), b.parameters()):
        if pa.grad is not None:
            torch.testing.assert_close(pa.grad, pb.grad)
    for s1, s2 in zip(sa, sb):
        for x, y in zip(s1.weights, s2.weights):
            torch.testing.assert_close(x, y)


@pytest.mark.parametrize("kind", ["mac", "mag"])
def test_in_place_weight_grad_accumulation_matches_autograd(kind):
    """Trainer backward (weight gradients added in place into the flat buffer) equals plain autograd."""
    import copy

    from titans_pytorch_b200.ops.linear import accumulate_weight_grads
    from titans_pytorch_b200.ops.loss import cross_entropy
    from titans_pytorch_b200.train.optim import FlatParamSpace

    a = tiny(kind)
    b = copy.deepcopy(a)
    ids = torch.randint(0, 64, (2, 41))
    loss_a = cross_entropy(a(ids[:, :-1])[0], ids[:, 1:])
    loss_a.backward()
    space = FlatParamSpace(b.parameters())
    space.zero_grad()
    with accumulate_weight_grads():
        cross_entropy(b(ids[:, :-1])[0], ids[:, 1:]).backward()
    for (n, pa), pb in zip(a.named_parameters(), b.parameters()):
        if pa.grad is None:
            continue
        torch.testing.assert_close(pb.grad, pa.grad, atol=1e-6, rtol=1e-5, msg=n)
    got = dict(zip([id(p) for p in space.params], space.got))
    assert all(got[id(p)] for p in b.parameters() if p.grad is not None and p.grad.abs().sum() > 0)


def test_p17_utilities():
    from titans_pytorch_b200.utils import perf as P

    torch.manual_seed(0)
    g, u = torch.randn(3, 8), torch.randn(3, 8)
    torch.testing.assert_close(P.fused_silu_mul(g, u), torch.nn.functional.silu(g) * u)
    x, r, w = torch.randn(2, 5, 16), torch.randn(2, 5, 16), torch.rand(16) + 0.5
    h, y = P.fused_add_rms_norm(x, r, w, 1e-6)
    torch.testing.assert_close(h, x + r)
    torch.testing.assert_close(y, (x + r) * torch.rsqrt((x + r).pow(2).mean(-1, keepdim=True) + 1e-6) * w)
    wg, wu, wd = torch.randn(32, 16) * 0.1, torch.randn(32, 16) * 0.1, torch.randn(16, 32) * 0.1
    torch.testing.assert_close(P.fused_linear_silu_linear(x, wg, wu, wd),
                               torch.nn.functional.linear(torch.nn.functional.silu(x @ wg.t()) * (x @ wu.t()), wd))
    with P.CUDAStreamManager(2).stream(1):
        pass
    m = tiny("mag").eval()
    ids = torch.randint(0, 64, (2, 6))
    logits, st = P.optimized_generate_step(m, ids)
    assert logits.shape == (2, 64) and len(st) == 2


def test_speculative_decode_equals_windowed_greedy():
    from titans_pytorch_b200.utils.perf import speculative_decode

    m = tiny("mag").eval()  # window 8 <= context 16
    draft = tiny("mag").eval()
    with torch.no_grad():
        for p in draft.parameters():
            p.add_(0.05 * torch.randn_like(p))  # a different (worse) draft
    ids = torch.randint(0, 64, (2, 20))
    got = speculative_decode(m, draft, ids, num_speculative_tokens=3, max_new_tokens=10, context=16)
    want = ids
    with torch.no_grad():
        for _ in range(10):
            lg, _ = m(want[:, -16:])
            want = torch.cat([want, lg[:, -1:].argmax(-1)], 1)
    assert torch.equal(got, want)
