"""titans_pytorch_b200: a Blackwell (sm_100a) framework for Titans neural-memory models.

The public names mirror the reference package's (`src/titans/__init__.py:19-111`)
so code written against it can switch by changing the import.
"""

from .config import ConfigError, TitansConfig
from .models import (FeedForward, MemoryMLP, MemoryState, NeuralLongTermMemory, PersistentMemory,
                     RMSNorm, RotaryPositionEmbedding, SegmentedAttention, SlidingWindowAttention,
                     TitansLMM, TitansMAC, TitansMAG, TitansMAL, create_model)

__version__ = "0.1.0"

__all__ = [
    "ConfigError", "TitansConfig", "FeedForward", "MemoryMLP", "MemoryState",
    "NeuralLongTermMemory", "PersistentMemory", "RMSNorm", "RotaryPositionEmbedding",
    "SegmentedAttention", "SlidingWindowAttention", "TitansLMM", "TitansMAC", "TitansMAG",
    "TitansMAL", "create_model",
]
