"""Oracle parity: this framework vs the reference package, fp32 on CPU.

The reference is imported read-only from ``baseline/_ref``.  Both sides get the
same weights (the reference's ``state_dict`` loaded strictly into ours), the
same tokens, and the reference's GPU memory-gradient semantics.
"""

from __future__ import annotations

import copy

import pytest
import torch
import torch.nn.functional as F

import titans_pytorch_b200 as T
from tests.conftest import import_reference, reference_cuda_semantics

VARIANTS = ["mac", "mag", "mal", "lmm"]


def _pair(monkeypatch, kind, **overrides):
    ref = import_reference()
    reference_cuda_semantics(monkeypatch, ref)
    fields = dict(dim=64, num_heads=4, num_layers=2, ffn_mult=2.0, num_memory_layers=2,
                  memory_hidden_mult=2.0, num_persistent_tokens=4, chunk_size=16,
                  window_size=8, dropout=0.0, vocab_size=100, max_seq_len=128)
    fields.update(overrides)
    torch.manual_seed(0)
    rcls = {"mac": ref.TitansMAC, "mag": ref.TitansMAG, "mal": ref.TitansMAL, "lmm": ref.TitansLMM}[kind]
    rm = rcls(ref.TitansConfig(**fields))
    om = T.create_model(kind, T.TitansConfig(**fields, use_kernels=False))
    om.load_state_dict(rm.state_dict(), strict=True)
    return rm, om


@pytest.mark.parametrize("kind", VARIANTS)
def test_state_dict_keys_and_order(monkeypatch, kind):
    rm, om = _pair(monkeypatch, kind)
    assert list(rm.state_dict().keys()) == list(om.state_dict().keys())
    for (k1, v1), (k2, v2) in zip(rm.state_dict().items(), om.state_dict().items()):
        assert v1.shape == v2.shape and v1.dtype == v2.dtype, k1


@pytest.mark.parametrize("kind", VARIANTS)
@pytest.mark.parametrize("mem_layers", [1, 2, 3])
def test_forward_backward_parity(monkeypatch, kind, mem_layers):
    rm, om = _pair(monkeypatch, kind, num_memory_layers=mem_layers)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 100, (2, 40), generator=g)
    labels = torch.randint(0, 100, (2, 40), generator=g)

    rl, rs = rm(ids)
    ol, os_ = om(ids)
    torch.testing.assert_close(ol, rl, atol=2e-5, rtol=1e-4)
    for a, b in zip(rs, os_):
        for x, y in zip(a.weights + a.momentum, b.weights + b.momentum):
            torch.testing.assert_close(y, x, atol=2e-6, rtol=1e-4)

    F.cross_entropy(rl.reshape(-1, 100), labels.reshape(-1)).backward()
    F.cross_entropy(ol.reshape(-1, 100), labels.reshape(-1)).backward()
    rp = dict(rm.named_parameters())
    for name, p in om.named_parameters():
        q = rp[name]
        assert (p.grad is None) == (q.grad is None), f"grad presence differs for {name}"
        if p.grad is not None:
            torch.testing.assert_close(p.grad, q.grad, atol=1e-5, rtol=1e-3, msg=name)


@pytest.mark.parametrize("kind", ["mac", "mag"])
def test_states_carry_and_param_writeback(monkeypatch, kind):
    """Two calls with carried states, and the parameter write-back of the memory state."""
    rm, om = _pair(monkeypatch, kind)
    ids = torch.randint(0, 100, (2, 24), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        rl1, rs = rm(ids)
        ol1, os_ = om(ids)
        rl2, _ = rm(ids, rs)
        ol2, _ = om(ids, os_)
        # a third call without states starts from whatever the parameters hold
        rl3, _ = rm(ids)
        ol3, _ = om(ids)
    torch.testing.assert_close(ol1, rl1, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(ol2, rl2, atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(ol3, rl3, atol=2e-5, rtol=1e-4)


def test_adamw_step_parity_tiny_mac(monkeypatch):
    """Tiny MAC (vocab 1000, dim 128, 2 layers, 4 heads, chunk 64, L_M=2), one AdamW step."""
    rm, om = _pair(monkeypatch, "mac", vocab_size=1000, dim=128, num_heads=4, num_layers=2,
                   num_persistent_tokens=4, chunk_size=64, num_memory_layers=2,
                   memory_hidden_mult=4.0, ffn_mult=4.0, conv_kernel_size=4)
    ids = torch.randint(0, 1000, (2, 257), generator=torch.Generator().manual_seed(0))
    x, y = ids[:, :-1], ids[:, 1:]
    ropt = torch.optim.AdamW(rm.parameters(), lr=4e-4, betas=(0.9, 0.95), weight_decay=0.1)
    oopt = torch.optim.AdamW(om.parameters(), lr=4e-4, betas=(0.9, 0.95), weight_decay=0.1)
    for m, opt in ((rm, ropt), (om, oopt)):
        logits, _ = m(x)
        F.cross_entropy(logits.reshape(-1, 1000), y.reshape(-1)).backward()
        torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0)
        opt.step()
    rp = dict(rm.named_parameters())
    for name, p in om.named_parameters():
        torch.testing.assert_close(p.detach(), rp[name].detach(), atol=1e-5, rtol=1e-4, msg=name)


def test_copy_of_reference_weights_is_loadable_by_reference(monkeypatch):
    ref = import_reference()
    rm, om = _pair(monkeypatch, "mag")
    rm2 = copy.deepcopy(rm)
    rm2.load_state_dict(om.state_dict(), strict=True)
    assert ref is not None
