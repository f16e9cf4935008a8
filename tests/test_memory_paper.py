"""Paper-semantics memory: the folded chunk recurrence, its gradient, and the model path (CPU)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import titans_pytorch_b200 as T
from titans_pytorch_b200.models.memory import _PaperScan
from titans_pytorch_b200.ops.memory_paper import (chunk_coefficients, head_blocks, memory_recurrence_tokenwise,
                                                  memory_scan_reference)


def _inputs(N, T_, d, hidden, L, seed=0):
    g = torch.Generator().manual_seed(seed)
    dims = [d] + [hidden] * (L - 1) + [d]
    W = [torch.randn(N, dims[i + 1], dims[i], generator=g) * 0.3 for i in range(L)]
    S = [torch.randn(w.shape, generator=g) * 0.1 for w in W]
    k = F.normalize(torch.randn(N, T_, d, generator=g), dim=-1)
    v = torch.randn(N, T_, d, generator=g)
    q = torch.randn(N, T_, d, generator=g)
    th = torch.sigmoid(torch.randn(N, T_, generator=g)) * 0.1
    et = torch.sigmoid(torch.randn(N, T_, generator=g)) * 0.9
    al = torch.sigmoid(torch.randn(N, T_, generator=g)) * 0.01
    return W, S, k, v, q, th, et, al


@pytest.mark.parametrize("L", [1, 2, 3])
def test_folded_chunk_update_equals_tokenwise_recurrence(L):
    W, S, k, v, q, th, et, al = _inputs(3, 70, 8, 16, L)
    _, Wn, Sn, _ = memory_scan_reference(W, S, k, v, None, th, et, al, 16)
    Wt, St = memory_recurrence_tokenwise(W, S, k, v, th, et, al, 16)
    for a, b in zip(Wn + Sn, Wt + St):
        assert ((a.double() - b).abs().max() / b.abs().max()) < 1e-5


def test_chunk_coefficients_edge_gates():
    C = 8
    th = torch.full((1, C), 0.3)
    # identity gates: no decay, full momentum
    A, b, c, p, d = chunk_coefficients(th, torch.ones(1, C), torch.zeros(1, C))
    assert torch.allclose(A, torch.ones(1)) and torch.allclose(p, torch.ones(1)) and torch.allclose(b, torch.full((1,), C * 1.0))
    # F_t = number of later steps + 1 when eta = 1, alpha = 0
    assert torch.allclose(c, 0.3 * torch.arange(C, 0, -1, dtype=torch.float32).unsqueeze(0))
    assert torch.allclose(d, th)
    # eta = 0: momentum forgets at every step (no NaN from log 0)
    A, b, c, p, d = chunk_coefficients(th, torch.zeros(1, C), torch.zeros(1, C))
    assert torch.isfinite(torch.cat([A, b, c.flatten(), p, d.flatten()])).all() and p.item() == 0.0


def test_scan_query_gradient_gradcheck():
    W, S, k, v, q, th, et, al = _inputs(2, 20, 4, 6, 2, seed=1)
    W, S = [w.double() for w in W], [s.double() for s in S]
    k, v = k.double(), v.double()
    qd = q.double().requires_grad_(True)

    def f(qq):
        return _PaperScan.apply(qq, k, v, th.double(), et.double(), al.double(), 8, "silu", False, 2, *W, *S)[0]

    assert torch.autograd.gradcheck(f, (qd,), eps=1e-6, atol=1e-5)


def test_head_blocks_layout():
    w = torch.arange(6 * 4, dtype=torch.float32).reshape(6, 4)
    blocks = head_blocks(w, 2)
    assert torch.equal(blocks[0], w[:3, :2]) and torch.equal(blocks[1], w[3:, 2:])


@pytest.mark.parametrize("kind", ["mac", "mag", "mal", "lmm"])
def test_paper_mode_models_train_and_carry_state(kind):
    cfg = T.TitansConfig(dim=64, num_heads=2, num_layers=2, vocab_size=100, chunk_size=32, window_size=16,
                         num_persistent_tokens=2, dropout=0.0, semantics="paper", memory_heads=2,
                         memory_chunk_size=16)
    torch.manual_seed(0)
    m = T.create_model(kind, cfg)
    ids = torch.randint(0, 100, (2, 50))
    logits, st = m(ids)
    assert st[0].weights[0].shape == (2, 2, cfg.memory_hidden_dim // 2, 32)
    logits.float().logsumexp(-1).mean().backward()
    assert m.layers[0].memory.proj_q.weight.grad is not None if hasattr(m, "layers") else True
    again, _ = m(ids, states=st)
    assert torch.isfinite(again).all() and not torch.allclose(again, logits)


def test_paper_mode_chunked_calls_match_one_call():
    """Feeding a sequence in chunk-aligned pieces with carried state equals one call (MAG)."""
    cfg = T.TitansConfig(dim=32, num_heads=2, num_layers=1, vocab_size=50, chunk_size=64, window_size=1 << 20,
                         num_persistent_tokens=0, dropout=0.0, semantics="paper", memory_heads=2,
                         memory_chunk_size=8, use_conv=False)
    torch.manual_seed(1)
    mem = T.NeuralLongTermMemory(cfg)
    x = torch.randn(2, 32, 32)
    full, s_full = mem(x)
    a, s = mem(x[:, :16])
    b, s = mem(x[:, 16:], state=s)
    torch.testing.assert_close(torch.cat([a, b], 1), full, atol=1e-5, rtol=1e-4)
    for w1, w2 in zip(s.weights, s_full.weights):
        torch.testing.assert_close(w1, w2, atol=1e-5, rtol=1e-4)
