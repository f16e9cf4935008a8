"""Persistent memory: N_p learnable, input-independent tokens prepended to attention.

Reference: `src/titans/persistent.py:25-73` (``tokens`` parameter ~ N(0, init_std),
batch-expanded view, ``None`` when N_p = 0).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ..config import TitansConfig


class PersistentMemory(nn.Module):
    def __init__(self, config: TitansConfig) -> None:
        super().__init__()
        self.config = config
        self.num_tokens = config.num_persistent_tokens
        self.dim = config.dim
        if self.num_tokens > 0:
            self.tokens = nn.Parameter(torch.randn(self.num_tokens, self.dim) * config.init_std)
        else:
            self.register_parameter("tokens", None)

    def forward(self, batch_size: int) -> torch.Tensor | None:
        if self.tokens is None:
            return None
        return self.tokens.unsqueeze(0).expand(batch_size, -1, -1)

    def get_tokens(self) -> torch.Tensor | None:
        return self.tokens
