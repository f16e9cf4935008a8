"""Incremental decoding (sliding-window KV ring + carried memory state) against
full forwards of the same model."""

from __future__ import annotations

import copy

import pytest
import torch

import titans_pytorch_b200 as T
from titans_pytorch_b200.inference.decode import StreamingDecoder, generate_incremental

FIELDS = dict(dim=64, num_heads=2, num_layers=2, vocab_size=128, window_size=8, chunk_size=16,
              num_persistent_tokens=4, dropout=0.0, max_seq_len=256, ffn_mult=2.0, memory_hidden_mult=2.0)


def _model(cls, **kw):
    torch.manual_seed(0)
    return getattr(T, cls)(T.TitansConfig(**{**FIELDS, **kw}, use_kernels=False)).eval()


@pytest.mark.parametrize("cls", ["TitansMAG", "TitansMAL", "TitansLMM"])
def test_decode_matches_prefix_forward_past_window(cls):
    """No memory update within the stream: every step equals the last position of
    a full forward over the prefix, including after the K/V ring wrapped 3 times."""
    model = _model(cls)
    oracle = copy.deepcopy(model)
    ids = torch.randint(0, 128, (2, 26), generator=torch.Generator().manual_seed(1))
    dec = StreamingDecoder(model, batch=2, update_every=10_000)
    for t in range(ids.shape[1]):
        got = dec.step(ids[:, t:t + 1])
        with torch.no_grad():
            ref = oracle(ids[:, :t + 1])[0][:, -1]
        torch.testing.assert_close(got, ref, atol=2e-4, rtol=2e-4, msg=f"position {t}")


@pytest.mark.parametrize("cls", ["TitansMAG", "TitansMAL", "TitansLMM"])
@pytest.mark.parametrize("L_M", [1, 2])
def test_decode_memory_update_matches_chunk_forward(cls, L_M):
    """After ``update_every`` tokens the carried states equal the new states of a
    forward over those tokens; decoding then continues from them."""
    model = _model(cls, num_memory_layers=L_M)
    oracle = copy.deepcopy(model)
    C = 16
    ids = torch.randint(0, 128, (2, C + 6), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        _, ref_states = oracle(ids[:, :C])
    dec = StreamingDecoder(model, batch=2, update_every=C)
    dec.prefill(ids[:, :C])
    for got, ref in zip(dec.states, ref_states, strict=True):
        for a, b in zip(got.weights + got.momentum, ref.weights + ref.momentum, strict=True):
            torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-4)
    outs = [dec.step(ids[:, t:t + 1]) for t in range(C, ids.shape[1])]
    assert all(torch.isfinite(o).all() for o in outs)
    # the same stream decoded again gives the same logits
    dec2 = StreamingDecoder(copy.deepcopy(oracle), batch=2, update_every=C)
    dec2.prefill(ids[:, :C])
    for t, o in zip(range(C, ids.shape[1]), outs):
        torch.testing.assert_close(dec2.step(ids[:, t:t + 1]), o)


def test_generate_incremental_greedy_matches_stepwise():
    model = _model("TitansMAG")
    prompt = torch.randint(0, 128, (1, 5), generator=torch.Generator().manual_seed(3))
    ids, states = generate_incremental(copy.deepcopy(model), prompt, max_new_tokens=6, greedy=True)
    assert ids.shape == (1, 11) and len(states) == FIELDS["num_layers"]
    dec = StreamingDecoder(model, batch=1)
    logits = dec.prefill(prompt)
    for t in range(6):
        nxt = logits.argmax(-1, keepdim=True)
        assert int(nxt) == int(ids[0, 5 + t])
        logits = dec.step(nxt)


def test_mac_is_refused():
    with pytest.raises(NotImplementedError):
        StreamingDecoder(_model("TitansMAC"))


@pytest.mark.gpu
def test_decode_bf16_kernels_match_prefix_forward():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.manual_seed(0)
    cfg = T.TitansConfig(**{**FIELDS, "dim": 128, "num_heads": 2, "window_size": 16})
    model = T.TitansMAG(cfg).cuda().to(torch.bfloat16).eval()
    oracle = copy.deepcopy(model)
    ids = torch.randint(0, 128, (2, 40), device="cuda")
    dec = StreamingDecoder(model, batch=2, update_every=10_000)
    for t in range(ids.shape[1]):
        got = dec.step(ids[:, t:t + 1]).float()
        with torch.no_grad():
            ref = oracle(ids[:, :t + 1])[0][:, -1].float()
        assert float((got - ref).norm() / ref.norm()) < 2e-2, t


# ------------------------------------------------------------------ int8 weights
def test_int8_model_matches_rounded_bf16_model_cpu():
    """Int8 weights (CPU path: dequantise on use) give the logits of a model whose
    weights were rounded to the same int8 grid; the bf16 storage is released."""
    from titans_pytorch_b200.inference.generate import quantize_model_dynamic
    from titans_pytorch_b200.ops.quant import Int8Weight, int8_weight_bytes, quantize_rows

    model = _model("TitansMAG")
    rounded = copy.deepcopy(model)
    with torch.no_grad():
        for m in rounded.modules():
            if isinstance(m, torch.nn.Linear) and m.bias is None and m.weight is not rounded.embed.weight:
                q, s = quantize_rows(m.weight)
                m.weight.copy_(q.float() * s[:, None])
    n_linear = sum(1 for m in model.modules() if isinstance(m, torch.nn.Linear) and m.bias is None)
    quantize_model_dynamic(model, bits=8)
    assert isinstance(model.head.weight, Int8Weight) and not isinstance(model.embed.weight, Int8Weight)
    assert not isinstance(model.blocks[0].memory.memory.layers[0].weight, Int8Weight)
    assert int8_weight_bytes(model) > 0 and n_linear > 0
    ids = torch.randint(0, 128, (2, 12), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        a = model(ids)[0]
        # the tied head of the rounded copy is the (unrounded) embedding: compare the hidden states
        b = rounded(ids)[0]
    ha = model.hidden_states(ids)[0]
    hb = rounded.hidden_states(ids)[0]
    torch.testing.assert_close(ha, hb, atol=1e-4, rtol=1e-4)
    assert a.shape == b.shape


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 16, 40])
def test_int8_gemm_vs_fp32(M):
    """int8 GEMM (M <= 16: in-register dequantisation; larger: transient bf16
    weight + tcgen05 GEMM) vs fp32 x @ (s q)^T."""
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from titans_pytorch_b200.ops.quant import Int8Weight, int8_linear, quantize_rows

    torch.manual_seed(0)
    N, K = 1000, 768
    w = (0.02 * torch.randn(N, K, device="cuda")).to(torch.bfloat16)
    q, s = quantize_rows(w)
    assert q.dtype == torch.int8 and s.dtype == torch.float32
    deq = q.float() * s[:, None]
    assert float((deq - w.float()).abs().max()) <= float(s.max()) * 0.5 + 1e-6
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = int8_linear(x, (Int8Weight(q, s),))
    ref = x.float() @ deq.t()
    assert float((y.float() - ref).norm() / ref.norm()) < 1e-2


@pytest.mark.gpu
def test_int8_decode_matches_bf16_decode():
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    from titans_pytorch_b200.ops.quant import quantize_model_int8

    torch.manual_seed(0)
    cfg = T.TitansConfig(**{**FIELDS, "dim": 128, "window_size": 16})
    model = T.TitansMAG(cfg).cuda().to(torch.bfloat16).eval()
    q = quantize_model_int8(copy.deepcopy(model))
    ids = torch.randint(0, 128, (2, 20), device="cuda")
    d0, d1 = StreamingDecoder(model, batch=2), StreamingDecoder(q, batch=2)
    for t in range(ids.shape[1]):
        a, b = d0.step(ids[:, t:t + 1]).float(), d1.step(ids[:, t:t + 1]).float()
        assert float((a - b).norm() / a.norm()) < 5e-2, t


@pytest.mark.gpu
def test_decode_graph_replay_matches_eager():
    """The captured step (device-side position, ring slot and mask; in-place
    buffers) replays the eager step, across memory updates."""
    if not torch.cuda.is_available():
        pytest.skip("needs CUDA")
    torch.manual_seed(0)
    cfg = T.TitansConfig(**{**FIELDS, "dim": 128, "window_size": 16})
    for cls in ("TitansMAG", "TitansMAL"):
        model = getattr(T, cls)(cfg).cuda().to(torch.bfloat16).eval()
        ids = torch.randint(0, 128, (2, 30), device="cuda")
        d0 = StreamingDecoder(model, batch=2, update_every=8)
        d1 = StreamingDecoder(model, batch=2, update_every=8, graph=True)
        for t in range(ids.shape[1]):
            a = d0.step(ids[:, t:t + 1]).float()
            b = d1.step(ids[:, t:t + 1]).float()
            assert float((a - b).abs().max()) <= 1e-3 * float(a.abs().max()) + 1e-3, (cls, t)
        for sa, sb in zip(d0.states, d1.states):
            for x, y in zip(sa.weights, sb.weights):
                torch.testing.assert_close(x.float(), y.float(), atol=1e-3, rtol=1e-2)
