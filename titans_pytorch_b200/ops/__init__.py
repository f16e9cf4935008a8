"""Operators: each runs an sm_100a kernel on CUDA tensors and a PyTorch restatement on CPU."""

from ._ext import available as kernels_available
from ._ext import want_kernels
from .attention import window_attention
from .conv import conv_silu_norm
from .ffn import swiglu_ffn
from .memory import memory_step
from .norm import rms_norm

__all__ = ["kernels_available", "want_kernels", "window_attention", "conv_silu_norm",
           "swiglu_ffn", "memory_step", "rms_norm"]
