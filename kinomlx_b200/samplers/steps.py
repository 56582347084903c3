"""Deterministic Euler steps of kinomlx/samplers/steps.py:8-70 on the device.

Same names, arguments, checks and rounding as the reference; each step is one elementwise
launch in libkino_b200.so (bf16 or fp32 CUDA tensors; nothing runs on the host).
"""

from __future__ import annotations

import math

import torch

from .. import ops, ops_f32


def euler_velocity_step(sample: torch.Tensor, velocity: torch.Tensor, sigma: float,
                        sigma_next: float) -> torch.Tensor:
    """sample + (fp32(sigma_next - sigma) * velocity in fp32, narrowed to the velocity dtype)
    (kinomlx/samplers/steps.py:8-33)."""
    if not math.isfinite(sigma) or not math.isfinite(sigma_next):
        raise ValueError("Euler velocity sigmas must be finite")
    if tuple(sample.shape) != tuple(velocity.shape):
        raise ValueError(
            f"velocity shape {tuple(velocity.shape)} does not match sample {tuple(sample.shape)}"
        )
    if sample.dtype != velocity.dtype:
        raise ValueError(
            f"velocity dtype {velocity.dtype} does not match sample dtype {sample.dtype}"
        )
    sample, velocity = sample.contiguous(), velocity.contiguous()
    if sample.dtype == torch.float32:
        delta = float(torch.tensor(sigma_next - sigma, dtype=torch.float32))
        return ops_f32.euler_velocity(sample, velocity, delta)
    return ops.euler_velocity_step(sample, velocity, sigma, sigma_next)


def euler_step(sample: torch.Tensor, denoised: torch.Tensor, sigma: float,
               sigma_next: float) -> torch.Tensor:
    """denoised + (sigma_next / sigma) * (sample - denoised) in fp32, returned in the sample's
    dtype (kinomlx/samplers/steps.py:36-70)."""
    if not math.isfinite(sigma) or sigma <= 0.0:
        raise ValueError(f"current sigma must be positive and finite, got {sigma!r}")
    if tuple(sample.shape) != tuple(denoised.shape):
        raise ValueError(
            f"denoised shape {tuple(denoised.shape)} does not match sample {tuple(sample.shape)}"
        )
    sample = sample.contiguous()
    if sample.dtype == torch.float32:
        return ops_f32.euler_denoised(sample, denoised.float().contiguous(), sigma, sigma_next)
    if denoised.dtype != sample.dtype:
        raise ValueError(f"denoised dtype {denoised.dtype} does not match sample {sample.dtype}")
    return ops.euler_denoised(sample, denoised.contiguous(), sigma, sigma_next)


__all__ = ["euler_step", "euler_velocity_step"]
