"""Deterministic-Euler denoising of the LTX-2 streams on the device
(kinomlx/models/ltx2/denoise.py:159-365, kinomlx/samplers/steps.py:36-70).

Two layers:
- `denoise_step` / `denoise_loop` keep the reference's signatures: latent states in, new latent
  states out (the caller's tensors are never written), the transformer as a keyword argument, a
  finiteness check after every step whose error names the stage or phase and the step;
- `denoise_video` / `denoise_video_step` are the bare loops the benchmark and the parity tests
  drive (one prepared context, the latent updated in place).

Each step is one X0 transformer evaluation with the Euler update fused into the final
projection's epilogue (x0 = x - sigma v, then x0 + (sigma'/sigma)(x - x0), both in fp32).

Supported here: uniform denoise masks (every token at the step's sigma), padded text masks on
the bf16 transformers (an additive key bias in the cross-attention), dense or Sol-Attn sparse
video self-attention (per step, video-only transformer on one GPU), the deterministic-Euler step.
The reference's other options (per-token masks from image/keyframe conditioning, keyframe masks,
the RF-ancestral step) are refused with a ValueError naming the option, never silently ignored.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass, replace

import torch

from .. import ops
from .transformer import LTXVideoTransformer, PreparedContext

# kinomlx/models/ltx2/sigmas.py:24-38: the distilled stage-1 schedule (9 values, 8 steps)
DISTILLED_STAGE_1_SIGMAS = (1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0)


def fp32(values) -> tuple[float, ...]:
    return tuple(float(torch.tensor(v, dtype=torch.float32)) for v in values)


class LTX2DenoiseError(RuntimeError):
    """A completed denoise step produced nonfinite active latents
    (kinomlx/models/ltx2/denoise.py:28-29)."""


@dataclass(frozen=True)
class LatentState:
    """kinomlx/models/ltx2/types.py:97-125: the latent being denoised, its per-token denoise
    mask, the positions of its tokens, the clean latent and whether every mask entry is 1."""

    latent: torch.Tensor
    denoise_mask: torch.Tensor | None
    positions: torch.Tensor
    clean_latent: torch.Tensor | None = None
    uniform_mask: bool = True


# ----------------------------------------------------------------------------- bare loops
def denoise_video_step(model: LTXVideoTransformer, prepared: PreparedContext, latent: torch.Tensor,
                       sigma: float, sigma_next: float) -> torch.Tensor:
    """One X0 transformer call and its Euler update, in place on `latent`."""
    if sigma <= 0:
        raise ValueError(f"current sigma must be positive, got {sigma!r}")
    return model.run(prepared, latent, sigma, sigma_next=sigma_next, out=latent)


def denoise_video(model: LTXVideoTransformer, latent: torch.Tensor, context: torch.Tensor,
                  positions: torch.Tensor, sigmas=DISTILLED_STAGE_1_SIGMAS,
                  check_finite: bool = True, context_mask=None) -> torch.Tensor:
    prepared = (model.prepare(context, positions) if context_mask is None
                else model.prepare(context, positions, context_mask=context_mask))
    t0, t1 = model.sp.shard(latent.shape[1])
    x = latent[:, t0:t1].to(model.device, getattr(model, "dtype", torch.bfloat16)).clone()
    values = fp32(sigmas)
    for s, n in zip(values[:-1], values[1:]):
        denoise_video_step(model, prepared, x, s, n)
    x = model.sp.all_gather_tokens(x)
    if check_finite:
        ops.device_status()
        if not bool(torch.isfinite(x).all()):
            raise FloatingPointError("LTX-2 denoising produced a nonfinite video latent")
    return x


# ----------------------------------------------------------------------------- reference surface
class _NullReporter:
    def phase_start(self, *args, **kwargs) -> None:
        pass

    def phase_advance(self, *args, **kwargs) -> None:
        pass

    def phase_end(self, *args, **kwargs) -> None:
        pass


def _refuse_unsupported(video_state: LatentState, audio_state: LatentState | None, *,
                        step_kind: str, video_context_mask, audio_context_mask,
                        video_keyframes_mask, video_noise, audio_noise, video_sparse_attention,
                        video_enabled: bool, audio_enabled: bool) -> None:
    if step_kind not in {"deterministic-euler", "ancestral-rf"}:
        raise ValueError(f"unknown denoise step kind {step_kind!r}")
    if step_kind != "deterministic-euler":
        raise ValueError("the device loop runs the deterministic Euler step only")
    if video_noise is not None or audio_noise is not None:
        raise ValueError("deterministic Euler must not receive transition noise")
    for state, name in ((video_state, "video"), (audio_state, "audio")):
        if state is not None and not state.uniform_mask:
            raise ValueError(f"the device loop takes uniform {name} denoise masks only")
    if audio_context_mask is not None and audio_state is None:
        raise ValueError("an audio text mask needs an audio latent state")
    if video_keyframes_mask is not None:
        raise ValueError("keyframe masks are not supported by the device loop")
    if video_sparse_attention is not None and audio_state is not None:
        raise ValueError("sparse video self-attention runs on the video-only transformer")
    if not video_enabled or not audio_enabled:
        raise ValueError("the device loop denoises every supplied modality")


def _check_finite(active: list[tuple[str, torch.Tensor]]) -> None:
    ops.device_status()
    for modality, value in active:
        if not bool(torch.isfinite(value).all()):
            raise LTX2DenoiseError(
                f"LTX-2 denoising produced a nonfinite {modality} latent in {value.dtype}.")


class _Prepared:
    """The once-per-loop preparation: context and RoPE tables for the transformer in use."""

    def __init__(self, transformer, video_state: LatentState, audio_state: LatentState | None,
                 video_context: torch.Tensor, audio_context: torch.Tensor | None,
                 video_context_mask=None, audio_context_mask=None):
        self.av = audio_state is not None
        if self.av:
            if audio_context is None:
                raise ValueError("audio context is required for an audio latent state")
            if not hasattr(transformer, "as_"):
                raise ValueError("an audio latent state needs the joint audio/video transformer")
            self.prep = transformer.prepare(video_context, audio_context, video_state.positions,
                                            audio_state.positions,
                                            video_context_mask=video_context_mask,
                                            audio_context_mask=audio_context_mask)
        elif video_context_mask is not None:
            self.prep = transformer.prepare(video_context, video_state.positions,
                                            context_mask=video_context_mask)
        else:
            self.prep = transformer.prepare(video_context, video_state.positions)


def _step(transformer, prepared: _Prepared, video_state: LatentState,
          audio_state: LatentState | None, sigma: float, sigma_next: float, sparse=None):
    dtype = getattr(transformer, "dtype", torch.bfloat16)
    video = video_state.latent.to(transformer.device, dtype)
    video_out = torch.empty_like(video)
    if prepared.av:
        audio = audio_state.latent.to(transformer.device, dtype)
        audio_out = torch.empty_like(audio)
        transformer.run(prepared.prep, video, audio, sigma, sigma_next=sigma_next,
                        video_out=video_out, audio_out=audio_out)
        active = [("video", video_out), ("audio", audio_out)]
        _check_finite(active)
        return replace(video_state, latent=video_out), replace(audio_state, latent=audio_out)
    sp = transformer.sp
    if sp.size > 1:  # each rank steps its token shard; the states carry whole latents
        t0, t1 = sp.shard(video.shape[1])
        shard = video[:, t0:t1].contiguous()
        transformer.run(prepared.prep, shard, sigma, sigma_next=sigma_next, out=shard)
        video_out = sp.all_gather_tokens(shard)
    else:
        kw = {} if sparse is None else {"sparse": sparse}
        transformer.run(prepared.prep, video, sigma, sigma_next=sigma_next, out=video_out, **kw)
    _check_finite([("video", video_out)])
    return replace(video_state, latent=video_out), audio_state


def denoise_step(
    video_state: LatentState,
    audio_state: LatentState | None,
    *,
    sigma: float,
    sigma_next: float,
    transformer,
    video_context: torch.Tensor,
    audio_context: torch.Tensor | None = None,
    video_context_mask: torch.Tensor | None = None,
    audio_context_mask: torch.Tensor | None = None,
    video_keyframes_mask: torch.Tensor | None = None,
    video_enabled: bool = True,
    audio_enabled: bool = True,
    step_kind: str = "deterministic-euler",
    video_noise: torch.Tensor | None = None,
    audio_noise: torch.Tensor | None = None,
    reporter=None,
    video_sparse_attention=None,
) -> tuple[LatentState, LatentState | None]:
    """One X0 transformer call and the Euler update of every supplied modality
    (kinomlx/models/ltx2/denoise.py:159-258); `transformer` is an LTXVideoTransformer, or an
    LTXAVTransformer when an audio state is given."""
    _refuse_unsupported(video_state, audio_state, step_kind=step_kind,
                        video_context_mask=video_context_mask,
                        audio_context_mask=audio_context_mask,
                        video_keyframes_mask=video_keyframes_mask, video_noise=video_noise,
                        audio_noise=audio_noise, video_sparse_attention=video_sparse_attention,
                        video_enabled=video_enabled, audio_enabled=audio_enabled)
    if not math.isfinite(sigma) or sigma <= 0.0:
        raise ValueError(f"current sigma must be positive and finite, got {sigma!r}")
    prepared = _Prepared(transformer, video_state, audio_state, video_context, audio_context,
                         video_context_mask, audio_context_mask)
    return _step(transformer, prepared, video_state, audio_state, fp32([sigma])[0],
                 fp32([sigma_next])[0], video_sparse_attention)


def denoise_loop(
    video_state: LatentState,
    audio_state: LatentState | None,
    sigmas: Sequence[float],
    *,
    transformer,
    video_context: torch.Tensor,
    audio_context: torch.Tensor | None = None,
    video_context_mask: torch.Tensor | None = None,
    audio_context_mask: torch.Tensor | None = None,
    video_keyframes_mask: torch.Tensor | None = None,
    reporter=None,
    phase: str = "denoise",
    callback: Callable[[int, int], None] | None = None,
    step_kind: str = "deterministic-euler",
    stage: int | None = None,
    noise_provider=None,
    video_sparse_attention: Sequence = (),
    transformer_dtype: torch.dtype | None = None,
) -> tuple[LatentState, LatentState | None]:
    """Run one sigma schedule (kinomlx/models/ltx2/denoise.py:261-365): the reference's schedule
    checks, one prepared context for the whole loop, a nonfinite step reported as
    "<stage or phase>, step <n>: ..."."""
    values = tuple(float(value) for value in sigmas)
    if len(values) < 2:
        raise ValueError("a denoise schedule must contain at least two sigmas")
    if any(not math.isfinite(current) or current <= 0.0 for current in values[:-1]):
        raise ValueError("every current denoise sigma must be positive and finite")
    if not math.isfinite(values[-1]):
        raise ValueError("the final denoise sigma must be finite")
    if any(current <= following for current, following in zip(values[:-1], values[1:])):
        raise ValueError("denoise sigmas must be strictly descending")
    if step_kind == "ancestral-rf" and stage is None:
        raise ValueError("ancestral RF needs the stage whose transition noise it draws")
    total = len(values) - 1
    if video_sparse_attention and len(video_sparse_attention) != total:
        raise ValueError(f"sparse attention lists {len(video_sparse_attention)} steps for a "
                         f"{total}-step schedule")
    sparse_steps = tuple(video_sparse_attention) or (None,) * total
    _refuse_unsupported(video_state, audio_state, step_kind=step_kind,
                        video_context_mask=video_context_mask,
                        audio_context_mask=audio_context_mask,
                        video_keyframes_mask=video_keyframes_mask, video_noise=None,
                        audio_noise=None,
                        video_sparse_attention=next((x for x in sparse_steps if x is not None), None),
                        video_enabled=True, audio_enabled=True)
    sink = reporter if reporter is not None else _NullReporter()
    prepared = _Prepared(transformer, video_state, audio_state, video_context, audio_context,
                         video_context_mask, audio_context_mask)
    schedule = fp32(values)
    sink.phase_start(phase, total=total, unit="step")
    try:
        for index in range(1, total + 1):
            try:
                video_state, audio_state = _step(transformer, prepared, video_state, audio_state,
                                                 schedule[index - 1], schedule[index],
                                                 sparse_steps[index - 1])
            except LTX2DenoiseError as error:
                location = f"stage {stage}" if stage is not None else phase
                message = f"{location}, step {index}: {error}"
                if transformer_dtype is not None and transformer_dtype == torch.float16:
                    message += (" The float16 transformer's activations may have overflowed;"
                                " select --transformer-dtype bfloat16 (or float32).")
                raise LTX2DenoiseError(message) from error
            sink.phase_advance(phase)
            if callback is not None:
                callback(index, total)
        return video_state, audio_state
    finally:
        sink.phase_end(phase)
