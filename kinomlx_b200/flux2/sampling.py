"""Klein Euler trajectory on the device (kinomlx/models/flux2/sampling.py:95-281).

Host work per step is scalar: the timestep's model-dtype round trip and dt, exactly as the
reference computes them. Without CFG the Euler update runs in the epilogue of the final
projection; with batched CFG the two velocities are combined by one elementwise kernel and the
update follows.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops, ops_f32
from .transformer import Flux2Transformer, PreparedText


def schedule(image_tokens: int, steps: int) -> torch.Tensor:
    """Empirical Klein shift (kinomlx/models/flux2/sampling.py:95-106), fp32."""
    if image_tokens < 1 or steps < 1:
        raise ValueError("Schedule requires positive target token and step counts")
    long = 0.00016927 * image_tokens + 0.45666666
    short = 8.73809524e-05 * image_tokens + 1.89833333
    mu = long if image_tokens > 4300 else long + (short - long) * (200 - steps) / 190
    factor = math.exp(mu)
    sigma = torch.tensor([1 - i / steps for i in range(steps)], dtype=torch.float32)
    shifted = factor / (factor + (1 / sigma - 1))
    return torch.cat([shifted, torch.zeros(1, dtype=torch.float32)])


def linear_sigmas(steps: int) -> torch.Tensor:
    """Explicit schedule linearly spaced from 1.0 to 0.0, fp32."""
    return torch.from_numpy(np.linspace(1.0, 0.0, steps + 1).astype(np.float32))


def timestep_x1000(sigmas: torch.Tensor, index: int, batch: int = 1,
                   dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """The value entering the timestep embedding: ((s*1000 -> dtype) / 1000 -> dtype) * 1000 ->
    dtype, with dtype the model's (kinomlx/models/flux2/sampling.py:209-212 and
    transformer.py:315); returned as fp32."""
    t = ((sigmas[index : index + 1] * 1000).to(dtype) / 1000).to(dtype)
    return (t * 1000).to(torch.float32).repeat(batch)


def step_delta(sigmas: torch.Tensor, index: int) -> float:
    """sigmas[i+1] - sigmas[i] in fp32 (kinomlx/models/flux2/sampling.py:240)."""
    return float(sigmas[index + 1] - sigmas[index])


def denoise_step(
    model: Flux2Transformer,
    prepared: PreparedText,
    current: torch.Tensor,
    sigmas: torch.Tensor,
    index: int,
    *,
    guidance: float = 1.0,
    cfg: bool = False,
    image: torch.Tensor | None = None,
) -> torch.Tensor:
    """One Euler step in place on `current` (1, Ni, C); returns `current`. The model's `dtype`
    (bf16, or fp32 for the parity-mode transformer) sets the timestep rounding and the
    elementwise kernels. `image` (1, Ni+Nr, C), when given, is the evaluated [target,
    reference] rows with `current` a view of its first Ni rows (sampling.py:255-281)."""
    dt = step_delta(sigmas, index)
    dtype = getattr(model, "dtype", torch.bfloat16)
    elementwise = ops_f32 if dtype == torch.float32 else ops
    # the timestep reaches the device as a fill value: a copy from pageable host memory would
    # wait for the stream to drain before every step
    t = float(timestep_x1000(sigmas, index, 1, dtype))
    rows = {} if image is None else {"target": (0, current.shape[1])}
    image = current if image is None else image
    if not cfg:
        return model.run(prepared, image, t, euler_dt=dt, sample=current, out=current, **rows)
    both = model.run(prepared, image.repeat(2, 1, 1), t, **rows)
    velocity = elementwise.cfg_combine(both[0:1], both[1:2], guidance)
    return elementwise.euler_velocity(current, velocity, dt, out=current)


def _finish(model, current: torch.Tensor, check_finite: bool) -> torch.Tensor:
    if check_finite:
        ops.device_status()
        if not bool(torch.isfinite(current).all()):
            raise FloatingPointError("Klein produced nonfinite latents")
    return current


def denoise(
    model: Flux2Transformer,
    noise: torch.Tensor,
    text: torch.Tensor,
    ids: torch.Tensor,
    *,
    sigmas: torch.Tensor,
    negative: torch.Tensor | None = None,
    guidance: float = 1.0,
    references: torch.Tensor | None = None,
    check_finite: bool = True,
) -> torch.Tensor:
    """Denoise `noise` (1, Ni, C) under `text` (1, Nt, C_txt); `ids` are the joint [text, image]
    positions (1, Nt+Ni, axes). Batched CFG when `negative` is given
    (kinomlx/models/flux2/sampling.py:116-281). With in-context `references` (1, Nr, C), every
    evaluation sees [target, reference] image rows, `ids` holds [text, target, reference]
    positions and only the target rows are updated (sampling.py:193-197, 264)."""
    if noise.dim() != 3 or noise.shape[0] != 1:
        raise ValueError("noise must be (1, tokens, channels)")
    if negative is not None and negative.shape != text.shape:
        raise ValueError("negative embeddings must match the positive text's shape")
    nr = 0 if references is None else references.shape[1]
    if references is not None:
        if references.dim() != 3 or references.shape[0] != 1 or nr < 1 \
                or references.shape[-1] != noise.shape[-1]:
            raise ValueError("Reference tokens and positions have incompatible shapes")
        if model.sp.size > 1:
            raise ValueError("in-context references run on one GPU")
    if ids.shape[1] != text.shape[1] + noise.shape[1] + nr:
        raise ValueError("Klein positions must match their token sequences")
    cfg = negative is not None and guidance != 1.0
    conditioned = text if not cfg else torch.cat([text, negative])
    prepared = model.prepare(conditioned, ids)
    dtype = getattr(model, "dtype", torch.bfloat16)
    i0, i1 = model.sp.shard(noise.shape[1])
    image = None
    if references is None:
        current = noise[:, i0:i1].to(model.device, dtype).clone()
    else:  # [target | reference] rows in one buffer; the Euler update writes the target rows
        image = torch.cat([noise, references], 1).to(model.device, dtype)
        current = image[:, : noise.shape[1]]
    for index in range(len(sigmas) - 1):
        denoise_step(model, prepared, current, sigmas, index, guidance=guidance, cfg=cfg,
                     image=image)
    current = model.sp.all_gather_tokens(current)
    return _finish(model, current.contiguous() if image is not None else current, check_finite)


def denoise_kv(
    model: Flux2Transformer,
    noise: torch.Tensor,
    text: torch.Tensor,
    text_ids: torch.Tensor,
    image_ids: torch.Tensor,
    references: torch.Tensor,
    reference_ids: torch.Tensor,
    *,
    sigmas: torch.Tensor,
    recompute_reference_kv: bool = False,
    check_finite: bool = True,
) -> torch.Tensor:
    """Klein KV editing (kinomlx/models/flux2/sampling.py:186-252): the first evaluation runs
    [reference, target] rows and keeps every layer's reference keys/values, the later ones run
    the target rows against the kept rows. With `recompute_reference_kv` each step extracts
    afresh. The cache is released when the loop ends, fails or is interrupted. No CFG (the
    reference's KV branch has none)."""
    if noise.dim() != 3 or noise.shape[0] != 1:
        raise ValueError("noise must be (1, tokens, channels)")
    if references.dim() != 3 or references.shape[0] != 1 or references.shape[1] < 1 \
            or references.shape[-1] != noise.shape[-1] \
            or tuple(reference_ids.shape[:2]) != (1, references.shape[1]):
        raise ValueError("Reference tokens and positions have incompatible shapes")
    if tuple(image_ids.shape[:2]) != (1, noise.shape[1]) \
            or tuple(text_ids.shape[:2]) != (1, text.shape[1]):
        raise ValueError("Klein positions must match their token sequences")
    if not hasattr(model, "new_reference_kv"):
        raise ValueError("this transformer has no reference K/V path")
    dtype = getattr(model, "dtype", torch.bfloat16)
    extract, reuse = model.prepare_layouts(
        text, (torch.cat([text_ids, reference_ids, image_ids], 1), torch.cat([text_ids, image_ids], 1)))
    nr = references.shape[1]
    # [reference | target] rows in one buffer: extraction reads all of it, reuse the target view
    image = torch.cat([references, noise], 1).to(model.device, dtype)
    current = image[:, nr:]
    cache = None
    try:
        for index in range(len(sigmas) - 1):
            dt = step_delta(sigmas, index)
            t = float(timestep_x1000(sigmas, index, 1, dtype))
            if cache is None:
                cache = model.new_reference_kv(nr)
            rows = image if cache.extracting else current
            model.run(extract if cache.extracting else reuse, rows, t, euler_dt=dt, sample=current,
                      out=current, reference_kv=cache)
            cache.extracting = False
            if recompute_reference_kv:
                cache.clear()
                cache = None
    finally:
        if cache is not None:
            cache.clear()
    return _finish(model, current.contiguous(), check_finite)
