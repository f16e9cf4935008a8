"""titans_pytorch_b200: a Blackwell (sm_100a) framework for Titans neural-memory models.

The public names mirror the reference package's (`src/titans/__init__.py:19-111`)
so code written against it can switch by changing the import.
"""

from .config import ConfigError, TitansConfig
from .inference.generate import (ContinuousBatcher, KVCacheConfig, OptimizedGenerator, StaticKVCache,
                                 benchmark_generation, generate)
from .models import (FeedForward, MemoryMLP, MemoryState, NeuralLongTermMemory, PersistentMemory,
                     RMSNorm, RotaryPositionEmbedding, SegmentedAttention, SlidingWindowAttention,
                     TitansLMM, TitansMAC, TitansMAG, TitansMAL, create_model)
from .train.optimized import OptimizedTrainer, OptimizedTrainingConfig, memory_efficient_attention
from .train.trainer import Trainer, TrainStepConfig
from .utils.checkpoint import load_checkpoint, load_model, save_checkpoint
from .utils.data import CUDAPrefetcher
from .utils.hub import load_from_hub, push_to_hub
from .utils.perf import (benchmark_model, compile_function, compile_model, enable_gradient_checkpointing,
                         get_optimal_batch_size, is_flash_attention_available, is_torch_sdpa_available,
                         is_triton_available)

# The reference's FlashAttention-2 wrappers are the same modules here: both attention
# forms already run on this framework's own flash kernels.
FlashSlidingWindowAttention = SlidingWindowAttention
FlashSegmentedAttention = SegmentedAttention

__version__ = "0.1.0"

__all__ = [
    "ConfigError", "TitansConfig", "MemoryState", "NeuralLongTermMemory", "MemoryMLP", "PersistentMemory",
    "SlidingWindowAttention", "SegmentedAttention", "FlashSlidingWindowAttention", "FlashSegmentedAttention",
    "RotaryPositionEmbedding", "FeedForward", "RMSNorm", "TitansMAC", "TitansMAG", "TitansMAL", "TitansLMM",
    "create_model", "is_flash_attention_available", "is_torch_sdpa_available", "is_triton_available",
    "push_to_hub", "load_from_hub", "save_checkpoint", "load_checkpoint", "load_model",
    "compile_model", "compile_function", "CUDAPrefetcher", "benchmark_model", "get_optimal_batch_size",
    "OptimizedTrainer", "OptimizedTrainingConfig", "enable_gradient_checkpointing", "memory_efficient_attention",
    "Trainer", "TrainStepConfig", "OptimizedGenerator", "StaticKVCache", "KVCacheConfig", "ContinuousBatcher",
    "benchmark_generation", "generate",
]
