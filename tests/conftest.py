"""Shared fixtures.  GPU tests carry ``@pytest.mark.gpu``; everything else runs on CPU."""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from titans_pytorch_b200.config import TitansConfig  # noqa: E402

REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running test")


def import_reference():
    """The reference package (installed read-only under baseline/_ref) or skip."""
    if not os.path.isdir(REF_DIR):
        pytest.skip("reference not installed under baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        import titans  # noqa: F401
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference import failed: {e}")
    return sys.modules["titans"]


def reference_cuda_semantics(monkeypatch, titans_mod):
    """Route the reference's memory gradient through its CUDA branch on CPU tensors.

    The reference picks its memory-gradient code by ``keys.is_cuda``
    (`src/titans/memory.py:310-320`); the GPU behaviour (memory MLP stays
    trainable, analytic L_M=1 form) is the one this framework implements.
    """
    from titans.cuda_optimizations import compute_memory_gradients_efficient

    fallback = titans_mod.memory.NeuralLongTermMemory._compute_gradients

    def _grads(self, keys, values):
        # same try/except shape as the reference's own CUDA dispatch
        try:
            weights = [layer.weight.data for layer in self.memory.layers]
            return compute_memory_gradients_efficient(keys.detach(), values.detach(), weights,
                                                      activation=self.config.activation)
        except Exception:
            return fallback(self, keys, values)

    monkeypatch.setattr(titans_mod.memory.NeuralLongTermMemory, "_compute_gradients", _grads)


@pytest.fixture
def default_config() -> TitansConfig:
    return TitansConfig(dim=64, num_heads=4, num_layers=2, ffn_mult=2.0, num_memory_layers=2,
                        memory_hidden_mult=2.0, num_persistent_tokens=4, num_memory_tokens=8,
                        chunk_size=32, window_size=16, dropout=0.0, use_conv=True,
                        conv_kernel_size=4, use_rope=True, max_seq_len=256, vocab_size=100)


@pytest.fixture
def small_config() -> TitansConfig:
    return TitansConfig(dim=32, num_heads=2, num_layers=1, ffn_mult=2.0, num_memory_layers=1,
                        memory_hidden_mult=2.0, num_persistent_tokens=2, num_memory_tokens=4,
                        chunk_size=16, window_size=8, dropout=0.0, use_conv=False,
                        use_rope=False, max_seq_len=64, vocab_size=50)


@pytest.fixture
def batch_size() -> int:
    return 2


@pytest.fixture
def seq_len() -> int:
    return 32


@pytest.fixture
def device() -> torch.device:
    return torch.device("cpu")


@pytest.fixture
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
