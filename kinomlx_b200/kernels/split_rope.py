"""`kinomlx.kernels.split_rope` surface (kinomlx/kernels/split_rope.py:139-166)."""

from __future__ import annotations

import torch

from .. import ops

_DTYPES = (torch.bfloat16,)
_enabled = True


def set_enabled(enabled: bool) -> None:
    global _enabled
    _enabled = bool(enabled)


def enabled() -> bool:
    return _enabled


def available(dtype: torch.dtype) -> bool:
    return dtype in _DTYPES


def applies(value: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor) -> bool:
    """Flattened-head (B, T, H*2*half) activations with fp32 head-major (B|1, H, T, half) tables."""
    if not _enabled or value.dim() != 3 or cos_freqs.dim() != 4:
        return False
    if cos_freqs.shape != sin_freqs.shape:
        return False
    if cos_freqs.dtype != torch.float32 or sin_freqs.dtype != torch.float32:
        return False
    table_batch, heads, tokens, half = cos_freqs.shape
    batch = value.shape[0]
    if table_batch not in (1, batch) or tuple(value.shape) != (batch, tokens, heads * 2 * half):
        return False
    return available(value.dtype) and value.is_cuda


def rotate(value: torch.Tensor, cos_freqs: torch.Tensor, sin_freqs: torch.Tensor) -> torch.Tensor:
    """Rotate each head's halves; bit-identical to the reference graph's fp32 products."""
    if not applies(value, cos_freqs, sin_freqs):
        raise ValueError("the RoPE kernel does not apply to these activations and tables")
    return ops.split_rope(value, cos_freqs, sin_freqs)
