"""Precision-policy ops of kinomlx/kernels/fused_ops.py:327-496 on the B200 kernels."""

from __future__ import annotations

import torch

from .. import ops


def gelu_approx(value: torch.Tensor) -> torch.Tensor:
    """tanh-GELU with fp32 opmath, input dtype preserved (kinomlx/kernels/fused_ops.py:327-350)."""
    return ops.gelu_tanh(value)


def silu(value: torch.Tensor) -> torch.Tensor:
    """SiLU with fp32 opmath (kinomlx/kernels/fused_ops.py:353-372)."""
    return ops.silu(value)


def rms_norm(
    value: torch.Tensor,
    weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    *,
    weight_offset: float = 0.0,
) -> torch.Tensor:
    """RMSNorm with fp32 reduction and scale, one rounding (kinomlx/kernels/fused_ops.py:412-457)."""
    if weight is not None and (weight.dim() != 1 or weight.shape[0] != value.shape[-1]):
        raise ValueError("rms_norm weight must be one-dimensional with the value's width")
    return ops.rms_norm(value.contiguous(), weight, eps, weight_offset=weight_offset)


def group_norm(value: torch.Tensor, norm) -> torch.Tensor:
    """Affine GroupNorm on channels-last input (kinomlx/kernels/fused_ops.py:375-409); `norm`
    carries num_groups, weight, bias and eps like the reference's nn.GroupNorm."""
    return ops.group_norm(value, norm.num_groups, norm.weight, norm.bias, norm.eps)


def pixel_norm(value: torch.Tensor, *, axis: int, eps: float) -> torch.Tensor:
    """Stepwise PixelNorm over the channel axis (kinomlx/kernels/fused_ops.py:460-476); the
    kernels take channels-last input, so `axis` must be the last one."""
    if axis not in (-1, value.dim() - 1):
        raise ValueError("pixel_norm runs over the last (channel) axis")
    return ops.pixel_norm(value, eps)


def pixel_norm_fp16(value: torch.Tensor, *, eps: float) -> torch.Tensor:
    """The reference's fused fp16 PixelNorm (kinomlx/kernels/fused_ops.py:486-493); bf16 is the
    supported activation type here, so this is the same kernel as `pixel_norm`."""
    if value.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("fused PixelNorm requires a channel-last low-precision array")
    return ops.pixel_norm(value, eps)
