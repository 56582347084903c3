"""Deterministic-Euler denoise loop for the LTX-2 video stream on the device
(kinomlx/models/ltx2/denoise.py:159-365, kinomlx/samplers/steps.py:36-70)."""

from __future__ import annotations

import torch

from .. import ops
from .transformer import LTXVideoTransformer, PreparedContext

# kinomlx/models/ltx2/sigmas.py:24-38: the distilled stage-1 schedule (9 values, 8 steps)
DISTILLED_STAGE_1_SIGMAS = (1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0)


def fp32(values) -> tuple[float, ...]:
    return tuple(float(torch.tensor(v, dtype=torch.float32)) for v in values)


def denoise_step(model: LTXVideoTransformer, prepared: PreparedContext, latent: torch.Tensor,
                 sigma: float, sigma_next: float) -> torch.Tensor:
    """One X0 transformer call and its Euler update, in place on `latent`."""
    if sigma <= 0:
        raise ValueError(f"current sigma must be positive, got {sigma!r}")
    return model.run(prepared, latent, sigma, sigma_next=sigma_next, out=latent)


def denoise_loop(model: LTXVideoTransformer, latent: torch.Tensor, context: torch.Tensor,
                 positions: torch.Tensor, sigmas=DISTILLED_STAGE_1_SIGMAS,
                 check_finite: bool = True) -> torch.Tensor:
    prepared = model.prepare(context, positions)
    t0, t1 = model.sp.shard(latent.shape[1])
    x = latent[:, t0:t1].to(model.device, getattr(model, "dtype", torch.bfloat16)).clone()
    values = fp32(sigmas)
    for s, n in zip(values[:-1], values[1:]):
        denoise_step(model, prepared, x, s, n)
    x = model.sp.all_gather_tokens(x)
    if check_finite:
        ops.device_status()
        if not bool(torch.isfinite(x).all()):
            raise FloatingPointError("LTX-2 denoising produced a nonfinite video latent")
    return x
