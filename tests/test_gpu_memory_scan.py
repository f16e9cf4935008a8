"""Fused chunked memory-scan kernel (sm_100a) against the fp32 PyTorch statement."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import titans_pytorch_b200 as T
from titans_pytorch_b200.ops import _ext
from titans_pytorch_b200.ops.memory_paper import memory_scan, memory_scan_reference

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("N,T_", [(1, 64), (3, 200), (5, 333), (130, 128)])
def test_memory_scan_kernel_matches_reference(N, T_):
    torch.manual_seed(3)
    d, hid = 64, 256
    W = [torch.randn(N, hid, d, device=DEV) * 0.05, torch.randn(N, d, hid, device=DEV) * 0.05]
    S = [torch.randn_like(w) * 0.01 for w in W]

    def unit():
        return F.normalize(torch.randn(N, T_, d, device=DEV), dim=-1).bfloat16()

    k, v, q = unit(), unit(), unit()
    th = torch.sigmoid(torch.randn(N, T_, device=DEV)) * 0.5
    et = torch.sigmoid(torch.randn(N, T_, device=DEV)) * 0.9
    al = torch.sigmoid(torch.randn(N, T_, device=DEV)) * 0.05
    E = _ext.ext()
    E.kernel_error_status(0, True)
    y, Wk, Sk = memory_scan(W, S, k, v, q, th, et, al, 64, use_kernels=True)
    torch.cuda.synchronize()
    assert E.kernel_error_status(0, True) == 0
    yr, Wr, Sr, _ = memory_scan_reference(W, S, k.float(), v.float(), q.float(), th, et, al, 64)
    assert rel(y, yr) < 2e-2
    for a, b in zip(Wk + Sk, Wr + Sr):
        assert rel(a, b) < 2e-2
    # the inputs were not modified in place
    assert torch.equal(W[0], W[0].clone())


def test_memory_scan_kernel_paper_model_matches_torch_path():
    cfg = T.TitansConfig(dim=128, num_heads=2, num_layers=2, vocab_size=256, chunk_size=128, window_size=64,
                         num_persistent_tokens=4, dropout=0.0, semantics="paper", memory_heads=2,
                         memory_chunk_size=64)
    torch.manual_seed(0)
    m = T.TitansMAG(cfg).to(DEV, torch.bfloat16)
    ids = torch.randint(0, 256, (2, 200), device=DEV)
    ref = T.TitansMAG(T.TitansConfig(**{**cfg.to_dict(), "use_kernels": False})).to(DEV, torch.bfloat16)
    ref.load_state_dict(m.state_dict())
    with torch.no_grad():
        a, sa = m(ids)
        b, sb = ref(ids)
    assert (a.float() - b.float()).abs().max().item() < 5e-2
    for x, y in zip(sa[0].weights, sb[0].weights):
        assert rel(x, y) < 3e-2
