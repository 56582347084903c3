"""Drop-in op surface of `kinomlx.kernels` (kinomlx/kernels/__init__.py:3) on the B200 kernels.

Same names and argument meaning as the reference, torch CUDA tensors in place of mx.array. Each
op is one launch in libkino_b200.so; there is no fallback path.
"""

from .fused_ops import gelu_approx, group_norm, pixel_norm, pixel_norm_fp16, rms_norm, silu

__all__ = ["gelu_approx", "group_norm", "pixel_norm", "pixel_norm_fp16", "rms_norm", "silu"]
