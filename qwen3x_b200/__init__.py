"""qwen3x_b200 -- B200 (sm_100a) kernels for qwen3x's packed-weight matrix path.

The compute lives in libq3xk.so (CUDA, built by `python -m qwen3x_b200.build`)
behind the C ABI of include/q3xk.h; this package is the host-side binding.
"""
from .capi import BF16, Q4_0, Q8_0, Q3xkError  # noqa: F401

__all__ = ["BF16", "Q8_0", "Q4_0", "Q3xkError"]
