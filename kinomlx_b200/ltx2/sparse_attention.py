"""Per-stage Sol-Attn schedules for LTX video self-attention
(kinomlx/models/ltx2/sparse_attention.py): the same schedule and dense-layer spellings, checks
and messages, and the per-step record a transformer forward takes.

A stage schedule gives each step a tau or ``dense``: ``dense``; ``auto`` (Sol-Engine's published
stage-2 taus 1, 1.25, 1.5; stage 2 only); one entry per step (or one for all), ``1,1.25,1.5``;
or step ranges ``5-8=1.5`` with the other steps dense. Dense layers are ``0,46-47`` or ``none``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..kernels.sol_attention import morton_order

DENSE = "dense"
AUTO = "auto"
AUTO_STAGE_2_TAUS: tuple[float, ...] = (1.0, 1.25, 1.5)
NO_LAYERS = "none"
LAYER_COUNT = 48

StepEntry = float | None  # a step's tau, or None for a dense step


def _entry(text: str) -> StepEntry:
    value = text.strip()
    if value == DENSE:
        return None
    try:
        tau = float(value)
    except ValueError:
        raise ValueError(f'a step takes a tau number or "{DENSE}", got {value!r}') from None
    if not math.isfinite(tau):
        raise ValueError(f"a step's tau must be finite, got {value!r}")
    return tau


def _step_range(text: str) -> tuple[int, int]:
    first, sep, last = text.strip().partition("-")
    try:
        start = int(first)
        end = int(last) if sep else start
    except ValueError:
        raise ValueError(f"steps are numbered from 1, like 3 or 5-8, got {text.strip()!r}") from None
    if start < 1 or end < start:
        raise ValueError(f"steps are numbered from 1, like 3 or 5-8, got {text.strip()!r}")
    return start, end


@dataclass(frozen=True)
class StepSchedule:
    """A parsed stage schedule: per-step entries, step ranges, or the auto schedule."""

    entries: tuple[StepEntry, ...] = ()
    ranges: tuple[tuple[int, int, StepEntry], ...] = ()
    auto: bool = False

    def resolve(self, steps: int, *, label: str, stage: int) -> tuple[StepEntry, ...]:
        if self.auto:
            if stage != 2:
                raise ValueError(f'{label}: "{AUTO}" is Sol-Engine\'s stage-2 schedule; stage 1 '
                                 f'takes taus or "{DENSE}"')
            if steps != len(AUTO_STAGE_2_TAUS):
                raise ValueError(f'{label}: "{AUTO}" sets the taus of the distilled three-step '
                                 f"stage 2 (1, 1.25 and 1.5), but the stage runs {steps} steps; "
                                 "write the taus out")
            return AUTO_STAGE_2_TAUS
        if self.ranges:
            out: list[StepEntry] = [None] * steps
            for start, end, entry in self.ranges:
                if end > steps:
                    raise ValueError(f"{label} names step {end}, but the stage runs {steps} steps")
                out[start - 1 : end] = [entry] * (end - start + 1)
            return tuple(out)
        if len(self.entries) == 1:
            return self.entries * steps
        if len(self.entries) != steps:
            raise ValueError(f"{label} lists {len(self.entries)} steps, but the stage runs {steps}; "
                             "give one entry per step or a single entry for every step")
        return self.entries


def parse_step_schedule(text: str) -> StepSchedule:
    """``dense``, ``auto``, ``1,1.25,1.5`` or ``5-8=1.5``."""
    if not isinstance(text, str) or not text.strip():
        raise ValueError(f'a sparse attention schedule must not be empty; use "{DENSE}"')
    if text.strip() == AUTO:
        return StepSchedule(auto=True)
    items = [item.strip() for item in text.split(",")]
    if any(not item for item in items):
        raise ValueError(f"a sparse attention schedule has an empty entry: {text!r}")
    keyed = ["=" in item for item in items]
    if not any(keyed):
        return StepSchedule(entries=tuple(_entry(item) for item in items))
    if not all(keyed):
        raise ValueError("a sparse attention schedule lists entries per step or sets STEPS=ENTRY "
                         f"items, not both: {text!r}")
    ranges: list[tuple[int, int, StepEntry]] = []
    for item in items:
        steps, _, entry = item.partition("=")
        start, end = _step_range(steps)
        for a, b, _ in ranges:
            if start <= b and a <= end:
                raise ValueError(f"a sparse attention schedule sets step {start} twice: {text!r}")
        ranges.append((start, end, _entry(entry)))
    return StepSchedule(ranges=tuple(sorted(ranges)))


def _render_entry(entry: StepEntry) -> str:
    return DENSE if entry is None else repr(entry).removesuffix(".0")


def canonical_step_schedule(text: str) -> str:
    """One spelling per schedule: entries joined by commas, ranges ascending as N or N-M."""
    schedule = parse_step_schedule(text)
    if schedule.auto:
        return AUTO
    if schedule.ranges:
        return ",".join((f"{a}" if a == b else f"{a}-{b}") + f"={_render_entry(e)}"
                        for a, b, e in schedule.ranges)
    return ",".join(_render_entry(e) for e in schedule.entries)


def is_dense_schedule(text: str) -> bool:
    """Whether a schedule leaves every step dense, whatever the step count."""
    schedule = parse_step_schedule(text)
    if schedule.auto:
        return False
    entries = [e for _, _, e in schedule.ranges] if schedule.ranges else schedule.entries
    return all(e is None for e in entries)


def parse_layer_ranges(text: str) -> tuple[int, ...]:
    """``0,46-47`` or ``none`` -> sorted distinct layer numbers."""
    if not isinstance(text, str) or not text.strip():
        raise ValueError(f'dense layers must not be empty; use "{NO_LAYERS}" for no layers')
    if text.strip() == NO_LAYERS:
        return ()
    layers: set[int] = set()
    for item in text.split(","):
        first, sep, last = item.strip().partition("-")
        try:
            start = int(first)
            end = int(last) if sep else start
        except ValueError:
            raise ValueError(f"dense layers are numbers and ranges like 0,46-47, got {item.strip()!r}") from None
        if not 0 <= start <= end < LAYER_COUNT:
            raise ValueError(f"dense layers run from 0 to {LAYER_COUNT - 1}, in increasing ranges, "
                             f"got {item.strip()!r}")
        span = set(range(start, end + 1))
        if layers & span:
            raise ValueError(f"dense layers repeat layer {min(layers & span)}")
        layers |= span
    return tuple(sorted(layers))


def render_layer_ranges(layers: tuple[int, ...]) -> str:
    """Sorted distinct layers as merged ranges, or ``none``."""
    if not layers:
        return NO_LAYERS
    runs: list[list[int]] = []
    for layer in layers:
        if runs and layer == runs[-1][1] + 1:
            runs[-1][1] = layer
        else:
            runs.append([layer, layer])
    return ",".join(f"{a}" if a == b else f"{a}-{b}" for a, b in runs)


def canonical_layer_ranges(text: str) -> str:
    return render_layer_ranges(parse_layer_ranges(text))


@dataclass(frozen=True)
class SparseAttentionSchedule:
    """One stage's resolved schedule: each step's tau or None, and the dense layers."""

    taus: tuple[StepEntry, ...]
    dense_layers: tuple[int, ...]

    @property
    def active(self) -> bool:
        return any(tau is not None for tau in self.taus)


def resolve_schedule(schedule: str, dense_layers: str, *, steps: int, label: str,
                     stage: int) -> SparseAttentionSchedule:
    taus = parse_step_schedule(schedule).resolve(steps, label=label, stage=stage)
    return SparseAttentionSchedule(taus, parse_layer_ranges(dense_layers))


@dataclass(frozen=True, eq=False)
class SparseAttentionStep:
    """Sparse video self-attention for one transformer forward: tau, the dense layers and the
    routing order of the video tokens (Morton order of the latent grid, then any appended
    tokens in their own order)."""

    tau: float
    dense_layers: frozenset[int]
    order: torch.Tensor

    def applies_to(self, layer: int) -> bool:
        return layer not in self.dense_layers


def stage_steps(schedule: SparseAttentionSchedule, *, grid: tuple[int, int, int],
                tokens: int) -> tuple[SparseAttentionStep | None, ...]:
    """Each step's forward record over a (frames, height, width) token grid."""
    if not schedule.active:
        return (None,) * len(schedule.taus)
    order = morton_order(*grid, tokens=tokens)
    dense = frozenset(schedule.dense_layers)
    return tuple(None if tau is None else SparseAttentionStep(tau, dense, order)
                 for tau in schedule.taus)


__all__ = ["AUTO", "AUTO_STAGE_2_TAUS", "DENSE", "LAYER_COUNT", "NO_LAYERS",
           "SparseAttentionSchedule", "SparseAttentionStep", "StepEntry", "StepSchedule",
           "canonical_layer_ranges", "canonical_step_schedule", "is_dense_schedule",
           "parse_layer_ranges", "parse_step_schedule", "render_layer_ranges",
           "resolve_schedule", "stage_steps"]
