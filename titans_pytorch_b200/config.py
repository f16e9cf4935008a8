"""Model configuration.

`TitansConfig` keeps the field names, defaults and derived properties of the
reference's config (`src/titans/config.py:10-107`) so that a checkpoint's
``config`` dict from either project constructs the same model here.  The
validation rules are the same; failures raise :class:`ConfigError`, which is
both a ``ValueError`` and an ``AssertionError`` so callers written against the
reference's ``assert``-based checks keep working.

Extra knobs (all optional, all with defaults that reproduce the reference):

* ``semantics`` -- ``"ref"`` reproduces the reference's memory behaviour
  (scalar gates averaged over batch/sequence/channels, one memory update per
  forward call, memory weights shared by the batch, parameter write-back of
  the memory state).  ``"paper"`` uses per-token gates and a chunked memory
  update with one memory per sample (the Titans paper's parallel form).
* ``memory_chunk_size`` -- chunk length of the paper-mode memory scan.
* ``memory_heads`` -- number of independent memories per sample in paper mode.
* ``use_kernels`` -- ``None`` (CUDA tensors run the sm_100a kernels, CPU
  tensors run the PyTorch restatement), ``True`` (require kernels),
  ``False`` (always the PyTorch restatement; used as the test oracle).
"""

from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any, Literal


class ConfigError(ValueError, AssertionError):
    """Invalid configuration value (catchable as ValueError or AssertionError)."""


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ConfigError(msg)


@dataclass
class TitansConfig:
    """Hyper-parameters of a Titans model.

    Field meanings follow the Titans paper: ``dim`` is d_in, ``num_memory_layers``
    is L_M (memory MLP depth), ``num_persistent_tokens`` is N_p,
    ``memory_lr``/``memory_momentum``/``memory_decay`` are the base scales of
    theta_t / eta_t / alpha_t.  ``memory_decay`` is accepted and validated but,
    as in the reference (`src/titans/memory.py:427-432`), the decay gate is the
    raw sigmoid mean and does not read it in ``ref`` semantics.
    """

    # Model dimensions
    dim: int = 512
    num_heads: int = 8
    num_layers: int = 12
    ffn_mult: float = 4.0

    # Memory
    num_memory_layers: int = 2
    memory_hidden_mult: float = 4.0
    num_persistent_tokens: int = 16
    num_memory_tokens: int = 64

    # Attention
    chunk_size: int = 512
    window_size: int = 512

    # Regularisation
    dropout: float = 0.1

    # Depthwise causal convolution after the memory projections
    use_conv: bool = True
    conv_kernel_size: int = 4

    # Positions
    use_rope: bool = True
    max_seq_len: int = 8192

    # Language modelling
    vocab_size: int = 32000

    # Memory learning rates
    memory_lr: float = 0.1
    memory_momentum: float = 0.9
    memory_decay: float = 0.01

    activation: Literal["silu", "gelu", "relu"] = "silu"
    init_std: float = 0.02

    # ---- knobs that have no reference counterpart -------------------------
    semantics: Literal["ref", "paper"] = "ref"
    memory_chunk_size: int = 64
    memory_heads: int = 1
    use_kernels: bool | None = field(default=None)
    norm_eps: float = 1e-6

    def __post_init__(self) -> None:
        _check(self.dim % self.num_heads == 0, "dim must be divisible by num_heads")
        _check(self.num_memory_layers >= 1, "num_memory_layers must be >= 1")
        _check(self.chunk_size > 0, "chunk_size must be positive")
        _check(self.window_size > 0, "window_size must be positive")
        _check(self.num_persistent_tokens >= 0, "num_persistent_tokens must be >= 0")
        _check(0.0 <= self.dropout < 1.0, "dropout must be in [0, 1)")
        _check(0.0 < self.memory_lr <= 1.0, "memory_lr must be in (0, 1]")
        _check(0.0 <= self.memory_momentum < 1.0, "memory_momentum must be in [0, 1)")
        _check(0.0 <= self.memory_decay < 1.0, "memory_decay must be in [0, 1)")
        _check(self.activation in ("silu", "gelu", "relu"), f"Unknown activation: {self.activation}")
        _check(self.semantics in ("ref", "paper"), "semantics must be 'ref' or 'paper'")
        _check(self.memory_chunk_size > 0, "memory_chunk_size must be positive")
        _check(self.memory_heads >= 1 and self.dim % self.memory_heads == 0,
               "memory_heads must divide dim")

    # Derived sizes (same definitions as the reference, config.py:94-107)
    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads

    @property
    def ffn_dim(self) -> int:
        return int(self.dim * self.ffn_mult)

    @property
    def memory_hidden_dim(self) -> int:
        return int(self.dim * self.memory_hidden_mult)

    # Serialisation -------------------------------------------------------
    def to_dict(self, reference_only: bool = False) -> dict[str, Any]:
        """Plain dict of the fields.

        ``reference_only=True`` drops the knobs the reference does not know, so
        the dict can be passed to the reference's ``TitansConfig(**d)``.
        """
        d = dataclasses.asdict(self)
        if reference_only:
            for k in _EXTRA_FIELDS:
                d.pop(k, None)
        return d

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "TitansConfig":
        """Build from a dict, ignoring unknown keys (e.g. a trainer's flags)."""
        names = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), indent=2, sort_keys=True)

    @classmethod
    def from_json(cls, s: str) -> "TitansConfig":
        return cls.from_dict(json.loads(s))

    @classmethod
    def from_file(cls, path: str) -> "TitansConfig":
        """Load a YAML or JSON file holding the config fields."""
        with open(path, encoding="utf-8") as f:
            text = f.read()
        if path.endswith((".yaml", ".yml")):
            import yaml

            return cls.from_dict(yaml.safe_load(text) or {})
        return cls.from_json(text)


_EXTRA_FIELDS = ("semantics", "memory_chunk_size", "memory_heads", "use_kernels", "norm_eps")
