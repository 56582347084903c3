"""Precision-policy ops of kinomlx/kernels/fused_ops.py restated on the CPU (test oracle)."""

from __future__ import annotations

import torch

LOW = (torch.bfloat16, torch.float16)


def gelu_approx(x: torch.Tensor) -> torch.Tensor:
    """tanh-GELU in fp32 opmath, inner argument clamped to +-10, one rounding
    (kinomlx/kernels/fused_ops.py:27-35, 327-350)."""
    f = x.float()
    inner = 0.7978845608028654 * (f + 0.044715 * f * f * f)
    return (0.5 * f * (1.0 + torch.tanh(inner.clamp(-10.0, 10.0)))).to(x.dtype)


def silu(x: torch.Tensor) -> torch.Tensor:
    """x / (1 + exp(-x)) in fp32, one rounding (kinomlx/kernels/fused_ops.py:40-45, 353-372)."""
    f = x.float()
    return (f / (1.0 + torch.exp(-f))).to(x.dtype)


def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    *,
    weight_offset: float = 0.0,
) -> torch.Tensor:
    """fp32 sum of squares, reciprocal root, fp32 scale by (weight + offset), one rounding
    (kinomlx/kernels/fused_ops.py:141-193, 412-457)."""
    f = x.float()
    inv = torch.rsqrt((f * f).mean(-1, keepdim=True) + eps)
    y = f * inv
    if weight is not None:
        y = y * (weight.float() + weight_offset)
    return y.to(x.dtype)


def layer_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """LayerNorm without affine, fp32 statistics, one rounding (mx.fast.layer_norm with no
    weight, used at kinomlx/models/flux2/transformer.py:57 and as nn.LayerNorm(affine=False) at
    kinomlx/models/ltx2/transformer/model.py:217)."""
    f = x.float()
    mean = f.mean(-1, keepdim=True)
    var = ((f - mean) ** 2).mean(-1, keepdim=True)
    return ((f - mean) * torch.rsqrt(var + eps)).to(x.dtype)


def pixel_norm(x: torch.Tensor, *, dim: int = -1, eps: float = 1e-8) -> torch.Tensor:
    """Stepwise square -> mean -> +eps -> sqrt -> divide in the value's dtype
    (kinomlx/kernels/fused_ops.py:460-476). Each step rounds to the input dtype; the mean
    accumulates in fp32 and rounds once."""
    dt = x.dtype
    sq = (x.float() * x.float()).to(dt)
    mean = sq.float().mean(dim, keepdim=True).to(dt)
    shifted = (mean.float() + eps).to(dt)
    rms = torch.sqrt(shifted.float()).to(dt)
    return (x.float() / rms.float()).to(dt)


def group_norm(
    x: torch.Tensor, groups: int, weight: torch.Tensor, bias: torch.Tensor, eps: float
) -> torch.Tensor:
    """Affine GroupNorm on channels-last input, fp32 two-pass statistics over each group's
    channels and all spatial positions, one rounding (kinomlx/kernels/fused_ops.py:47-139,
    375-409)."""
    dt = x.dtype
    shape = x.shape
    c = shape[-1]
    f = x.float().reshape(shape[0], -1, groups, c // groups)
    mean = f.mean(dim=(1, 3), keepdim=True)
    var = ((f - mean) ** 2).mean(dim=(1, 3), keepdim=True)
    y = ((f - mean) * torch.rsqrt(var + eps)).reshape(shape)
    return (y * weight.float() + bias.float()).to(dt)


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """addmm with an (out, in) weight: fp32 accumulation, bias added to the fp32 sum, one
    rounding to the activation dtype (kinomlx/kernels/mpp_linear.py:1-11: mx.addmm's epilogue;
    kinomlx/modeling/layers.py:8-31)."""
    y = x.float() @ w.float().T
    if b is not None:
        y = y + b.float()
    return y.to(x.dtype)


def linear_then_bias(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """A packed (quantised) linear: the matmul rounded to the activation dtype, then the bias added
    as a separate bf16 operation (kinomlx/models/ltx2/weights/quantization.py:32-43:
    `mx.quantized_matmul(...)` then `result + bias`)."""
    y = (x.float() @ w.float().T).to(x.dtype)
    if b is not None:
        y = (y.float() + b.float()).to(x.dtype)
    return y


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
         mask: torch.Tensor | None = None) -> torch.Tensor:
    """Scaled dot-product attention on (B, H, T, D) in fp32, one rounding
    (mx.fast.scaled_dot_product_attention at kinomlx/models/flux2/kv.py:48-54); an additive
    `mask` broadcastable to (B, H, Tq, Tk) is added to the scaled scores
    (kinomlx/models/ltx2/transformer/attention.py:164-186)."""
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if mask is not None:
        s = s + mask.float()
    return (torch.softmax(s, dim=-1) @ v.float()).to(q.dtype)
