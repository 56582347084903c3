"""Klein Euler trajectory on the device (kinomlx/models/flux2/sampling.py:95-281).

Host work per step is scalar: the timestep's model-dtype round trip and dt, exactly as the
reference computes them. Without CFG the Euler update runs in the epilogue of the final
projection; with batched CFG the two velocities are combined by one elementwise kernel and the
update follows.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from dataclasses import dataclass
from enum import Enum

import numpy as np
import torch

from .. import ops, ops_f32
from .transformer import Flux2Transformer, PreparedText


class Flux2Variant(str, Enum):
    """Klein checkpoint profiles (kinomlx/models/flux2/catalog.py:7-32)."""

    BASE = "base"
    DISTILLED = "distilled"
    KV = "kv"


class Flux2CFGMode(str, Enum):
    """How the two guidance branches are evaluated (kinomlx/models/flux2/request_constraints.py:12-17)."""

    SEQUENTIAL = "sequential"
    BATCHED = "batched"


# variant -> (default steps, default guidance, reference K/V) (catalog.py:26-30)
_PROFILES = {
    Flux2Variant.BASE: (50, 4.0, False),
    Flux2Variant.DISTILLED: (4, 1.0, False),
    Flux2Variant.KV: (4, 1.0, True),
}


def _validated_sigmas(values) -> tuple[float, ...]:
    """kinomlx/samplers/sigmas.py:48-80 (SigmaSchedule): at least two finite values inside
    [0, 1], strictly decreasing."""
    values = tuple(float(value) for value in values)
    if len(values) < 2:
        raise ValueError("a sigma schedule needs at least two values, one more than its step count")
    if any(not math.isfinite(value) for value in values):
        raise ValueError("sigma values must be finite")
    outside = [f"{value:g}" for value in values if not 0.0 <= value <= 1.0]
    if outside:
        raise ValueError(f"sigma values must lie between 0 and 1, got {', '.join(outside)}")
    if any(a <= b for a, b in zip(values[:-1], values[1:])):
        raise ValueError("sigma values must decrease strictly, got "
                         + ", ".join(f"{value:g}" for value in values))
    return values


@dataclass(frozen=True)
class SamplingRecipe:
    """kinomlx/models/flux2/sampling.py:53-96 and recipe_rules.py:8-44: the variant's profile
    supplies the step count and guidance unless given; explicit `sigmas` own the step count."""

    variant: Flux2Variant = Flux2Variant.DISTILLED
    steps: int | None = None
    guidance: float | None = None
    cfg_mode: Flux2CFGMode = Flux2CFGMode.SEQUENTIAL
    recompute_reference_kv: bool = False
    sigmas: tuple[float, ...] = ()

    @property
    def explicit_sigmas(self) -> bool:
        return bool(self.sigmas)

    def resolved(self) -> tuple[int, float]:
        variant = Flux2Variant(self.variant)
        default_steps, default_guidance, kv = _PROFILES[variant]
        if self.steps is not None and self.steps < 1:
            raise ValueError("steps must be at least 1")
        if self.guidance is not None and self.guidance < 1:
            raise ValueError("guidance must be at least 1")
        if self.sigmas:
            _validated_sigmas(self.sigmas)
        if self.recompute_reference_kv and not kv:
            raise ValueError("Reference K/V recomputation requires the KV recipe")
        steps = len(self.sigmas) - 1 if self.sigmas else default_steps if self.steps is None else self.steps
        guidance = default_guidance if self.guidance is None else float(self.guidance)
        if variant != Flux2Variant.BASE:
            if guidance != 1:
                raise ValueError("External CFG is supported by the base recipe only")
            if Flux2CFGMode(self.cfg_mode) != Flux2CFGMode.SEQUENTIAL:
                raise ValueError("cfg_mode batched requires the base model")
        return steps, guidance

    def sigma_array(self, image_tokens: int) -> torch.Tensor:
        """The explicit schedule, else the Klein shift; validated either way, fp32."""
        values = self.sigmas or tuple(float(v) for v in schedule(image_tokens, self.resolved()[0]))
        try:
            return torch.tensor(_validated_sigmas(values), dtype=torch.float32)
        except ValueError as exc:
            raise ValueError(f"Klein schedule: {exc}") from exc


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


def euler_step(current: torch.Tensor, velocity: torch.Tensor, delta) -> torch.Tensor:
    """dt rounded to the model dtype times the velocity in the model dtype, added to the fp32
    sample (kinomlx/models/flux2/sampling.py:109-113); one elementwise launch."""
    dt = float(torch.as_tensor(delta, dtype=torch.float32))
    if current.dtype == torch.float32:
        return ops_f32.euler_velocity(current.contiguous(), velocity.contiguous(), dt)
    return ops.euler_velocity(current.contiguous(), velocity.contiguous(), dt)


def _finish(model, current: torch.Tensor, check_finite: bool) -> torch.Tensor:
    if check_finite:
        ops.device_status()
        if not bool(torch.isfinite(current).all()):
            raise FloatingPointError("Klein produced nonfinite latents")
    return current


class _NullReporter:
    def phase_start(self, *args, **kwargs) -> None:
        pass

    def phase_advance(self, *args, **kwargs) -> None:
        pass

    def phase_end(self, *args, **kwargs) -> None:
        pass


def _finite(value: torch.Tensor | None) -> bool:
    return value is None or bool(torch.isfinite(value).all())


def denoise(
    model: Flux2Transformer,
    noise: torch.Tensor,
    text: torch.Tensor,
    image_ids: torch.Tensor,
    text_ids: torch.Tensor,
    *,
    recipe: SamplingRecipe | None = None,
    references: torch.Tensor | None = None,
    reference_ids: torch.Tensor | None = None,
    negative: torch.Tensor | None = None,
    reporter=None,
    on_step: Callable[[int, torch.Tensor, torch.Tensor], None] | None = None,
) -> torch.Tensor:
    """The reference's Klein loop with its signature, checks and errors
    (kinomlx/models/flux2/sampling.py:116-281). Shapes are the model's: noise (1, Ni, in_channels),
    text (1, Nt, context_dim), ids (1, N, len(rope_axes)). Per step: the evaluation (KV
    extraction or reuse; in-context references; batched CFG as one batch-2 evaluation or
    sequential CFG as two), the Euler update and a finiteness check that names the step;
    `on_step(index, current, velocity)` sees every step's velocity (the velocity is then
    materialised and the update runs as its own launch instead of in the final projection's
    epilogue; the result is the same). Supplied conditioning is never mutated."""
    recipe = recipe or SamplingRecipe()
    steps, guidance = recipe.resolved()
    v = model.v
    axes = len(v.rope_axes)
    if noise.dim() != 3 or noise.shape[0] != 1 or noise.shape[-1] != v.in_channels:
        raise ValueError(f"Klein noise requires [1, target tokens, {v.in_channels}]")
    if text.dim() != 3 or text.shape[0] != 1 or text.shape[-1] != v.context_dim:
        raise ValueError(f"Klein text requires [1, text tokens, {v.context_dim}]")
    if tuple(image_ids.shape) != (1, noise.shape[1], axes) or tuple(text_ids.shape) != (1, text.shape[1], axes):
        raise ValueError("Klein positions must match their token sequences")
    if (references is None) != (reference_ids is None):
        raise ValueError("References and reference positions must be supplied together")
    if references is not None and (
        references.dim() != 3 or references.shape[0] != 1 or references.shape[1] < 1
        or references.shape[-1] != v.in_channels
        or tuple(reference_ids.shape) != (1, references.shape[1], axes)
    ):
        raise ValueError("Reference tokens and positions have incompatible shapes")
    if guidance > 1 and negative is None:
        raise ValueError(
            "Base CFG requires explicit negative embeddings (encode empty text for default CFG)")
    if negative is not None and (guidance == 1 or negative.shape != text.shape):
        raise ValueError(
            "Negative embeddings require active CFG and the same shape as positive text")
    if noise.dtype not in (torch.float16, torch.bfloat16, torch.float32) or any(
            value is not None and value.dtype != noise.dtype for value in (text, references, negative)):
        raise ValueError("Klein noise and conditioning require a common FP16, BF16, or FP32 dtype")
    if not all(_finite(value) for value in (noise, text, references, negative, image_ids, text_ids,
                                            reference_ids)):
        raise ValueError("Klein conditioning and noise must be finite")
    sigmas = recipe.sigma_array(noise.shape[1])
    dtype = getattr(model, "dtype", torch.bfloat16)
    elementwise = ops_f32 if dtype == torch.float32 else ops
    progress = reporter or _NullReporter()
    kv_edit = Flux2Variant(recipe.variant) == Flux2Variant.KV and references is not None
    batched = negative is not None and Flux2CFGMode(recipe.cfg_mode) == Flux2CFGMode.BATCHED
    sequential = negative is not None and not batched
    if (kv_edit or references is not None) and model.sp.size > 1:
        raise ValueError("in-context references run on one GPU")
    ni, nr = noise.shape[1], 0 if references is None else references.shape[1]
    cache = None
    progress.phase_start("denoise", total=steps, unit="step")
    try:
        if kv_edit:
            extract, reuse = model.prepare_layouts(
                text, (torch.cat([text_ids, reference_ids, image_ids], 1),
                       torch.cat([text_ids, image_ids], 1)))
            image = torch.cat([references, noise], 1).to(model.device, dtype)
            current = image[:, nr:]
        else:
            ids = torch.cat([text_ids, image_ids] + ([] if references is None else [reference_ids]), 1)
            predict = model.prepare(torch.cat([text, negative]) if batched else text, ids)
            negative_predict = model.prepare(negative, ids) if sequential else None
            i0, i1 = model.sp.shard(ni)
            if references is None:
                image = None
                current = noise[:, i0:i1].to(model.device, dtype).clone()
            else:
                image = torch.cat([noise, references], 1).to(model.device, dtype)
                current = image[:, :ni]
        rows = {} if references is None or kv_edit else {"target": (0, ni)}
        kept = torch.empty_like(current) if sequential or on_step is not None else None
        for index in range(steps):
            dt = step_delta(sigmas, index)
            t = float(timestep_x1000(sigmas, index, 1, dtype))
            velocity = None
            if kv_edit:
                if cache is None:
                    cache = model.new_reference_kv(nr)
                evaluated = image if cache.extracting else current
                layout = extract if cache.extracting else reuse
                if on_step is None:
                    model.run(layout, evaluated, t, euler_dt=dt, sample=current, out=current,
                              reference_kv=cache)
                else:
                    velocity = model.run(layout, evaluated, t, out=kept, reference_kv=cache)
                cache.extracting = False
                if recipe.recompute_reference_kv:
                    cache.clear()
                    cache = None
            else:
                evaluated = current if image is None else image
                if batched:
                    both = model.run(predict, evaluated.repeat(2, 1, 1), t, **rows)
                    velocity = elementwise.cfg_combine(both[0:1], both[1:2], guidance)
                elif sequential:
                    positive = model.run(predict, evaluated, t, out=kept, **rows)
                    uncond = model.run(negative_predict, evaluated, t, **rows)
                    velocity = elementwise.cfg_combine(positive, uncond, guidance)
                elif on_step is not None:
                    velocity = model.run(predict, evaluated, t, out=kept, **rows)
                else:
                    model.run(predict, evaluated, t, euler_dt=dt, sample=current, out=current, **rows)
            if velocity is not None:
                elementwise.euler_velocity(current, velocity, dt, out=current)
            ops.device_status()
            if not bool(torch.isfinite(current).all()):
                raise FloatingPointError(f"Klein produced nonfinite latents at step {index + 1}")
            progress.phase_advance("denoise")
            if on_step is not None:
                on_step(index, current, velocity)
    finally:
        if cache is not None:
            cache.clear()
        progress.phase_end("denoise")
    if not kv_edit:
        current = model.sp.all_gather_tokens(current)
    return current.contiguous()


def denoise_joint(
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
