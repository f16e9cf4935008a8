"""Titans model family: modules and the four model variants."""

from .attention import RotaryPositionEmbedding, SegmentedAttention, SlidingWindowAttention
from .layers import FeedForward, RMSNorm
from .memory import MemoryMLP, MemoryState, NeuralLongTermMemory, get_activation
from .persistent import PersistentMemory
from .titans import (MODEL_CLASSES, LMMBlock, MACBlock, MAGBlock, MALBlock, TitansLMM, TitansMAC,
                     TitansMAG, TitansMAL, create_model)

__all__ = [
    "RotaryPositionEmbedding", "SegmentedAttention", "SlidingWindowAttention", "FeedForward",
    "RMSNorm", "MemoryMLP", "MemoryState", "NeuralLongTermMemory", "get_activation",
    "PersistentMemory", "MODEL_CLASSES", "LMMBlock", "MACBlock", "MAGBlock", "MALBlock",
    "TitansLMM", "TitansMAC", "TitansMAG", "TitansMAL", "create_model",
]
