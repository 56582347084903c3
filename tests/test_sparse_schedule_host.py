"""The Sol-Attn schedule host logic (kinomlx_b200.ltx2.sparse_attention) pinned against the
known answers of the reference's schedule tests (tests/models/ltx2/test_sparse_attention_schedule.py:
resolution per step, the refusals and their messages, auto, canonical spellings, dense layers),
and the per-step records `stage_steps` builds for a latent grid."""

from __future__ import annotations

import pytest
import torch

from kinomlx_b200.kernels.sol_attention import morton_order
from kinomlx_b200.ltx2.sparse_attention import (AUTO_STAGE_2_TAUS, SparseAttentionSchedule,
                                                canonical_layer_ranges, canonical_step_schedule,
                                                is_dense_schedule, parse_layer_ranges,
                                                parse_step_schedule, resolve_schedule, stage_steps)


@pytest.mark.parametrize(("text", "steps", "expected"), [
    ("dense", 3, (None, None, None)),
    ("1.5", 3, (1.5, 1.5, 1.5)),
    ("1,1.25,1.5", 3, (1.0, 1.25, 1.5)),
    ("dense,1,dense", 3, (None, 1.0, None)),
    ("5-8=1.5", 8, (None, None, None, None, 1.5, 1.5, 1.5, 1.5)),
    ("2=1, 4-5=0.75,7-7=dense", 8, (None, 1.0, None, 0.75, 0.75, None, None, None)),
    ("1-3=-0.5", 3, (-0.5, -0.5, -0.5)),
])
def test_schedules_resolve_each_step(text, steps, expected):
    assert parse_step_schedule(text).resolve(steps, label="schedule", stage=1) == expected


@pytest.mark.parametrize(("text", "message"), [
    ("", "must not be empty"), ("  ", "must not be empty"), ("1,,2", "empty entry"),
    ("1,x", 'tau number or "dense"'), ("inf", "must be finite"), ("nan", "must be finite"),
    ("1,2=1.5", "not both"), ("0=1", "numbered from 1"), ("3-2=1", "numbered from 1"),
    ("a-2=1", "numbered from 1"), ("1-3=1,3=2", "sets step 3 twice"),
])
def test_malformed_schedules_fail_with_the_reason(text, message):
    with pytest.raises(ValueError, match=message):
        parse_step_schedule(text)


def test_step_counts_auto_and_spellings():
    with pytest.raises(ValueError, match="lists 2 steps, but the stage runs 3"):
        parse_step_schedule("1,2").resolve(3, label="stage_2_sparse_attention", stage=2)
    with pytest.raises(ValueError, match="names step 5, but the stage runs 3"):
        parse_step_schedule("2-5=1").resolve(3, label="stage_2_sparse_attention", stage=2)
    assert AUTO_STAGE_2_TAUS == (1.0, 1.25, 1.5)
    auto = parse_step_schedule(" auto ")
    assert auto.resolve(3, label="s", stage=2) == AUTO_STAGE_2_TAUS
    assert canonical_step_schedule(" auto ") == "auto" and not is_dense_schedule("auto")
    with pytest.raises(ValueError, match="stage-2 schedule; stage 1 takes taus"):
        auto.resolve(8, label="s", stage=1)
    with pytest.raises(ValueError, match="but the stage runs 4 steps; write the taus out"):
        auto.resolve(4, label="s", stage=2)
    with pytest.raises(ValueError, match="tau number"):
        parse_step_schedule("auto,1")
    for text, canonical in ((" 1, 1.25 ,1.50 ", "1,1.25,1.5"), ("dense, 2.0", "dense,2"),
                            ("dense,dense", "dense,dense"),
                            ("7-8=1.5,1=dense, 3-3=1", "1=dense,3=1,7-8=1.5"), ("1e-1", "0.1")):
        assert canonical_step_schedule(text) == canonical
        assert canonical_step_schedule(canonical) == canonical
    assert is_dense_schedule("dense") and is_dense_schedule("dense,dense,dense")
    assert is_dense_schedule("1-8=dense")
    assert not is_dense_schedule("dense,1") and not is_dense_schedule("8=1.5")


@pytest.mark.parametrize(("text", "layers", "canonical"), [
    ("0", (0,), "0"), ("none", (), "none"), ("47, 0,46", (0, 46, 47), "0,46-47"),
    ("0-3,5", (0, 1, 2, 3, 5), "0-3,5"), ("0,1,2", (0, 1, 2), "0-2"),
    ("0-47", tuple(range(48)), "0-47"),
])
def test_dense_layers_take_numbers_and_ranges(text, layers, canonical):
    assert parse_layer_ranges(text) == layers
    assert canonical_layer_ranges(text) == canonical


def test_stage_steps_records():
    schedule = resolve_schedule("dense,1.25,1.5", "0,46-47", steps=3, label="s", stage=2)
    assert schedule == SparseAttentionSchedule((None, 1.25, 1.5), (0, 46, 47))
    steps = stage_steps(schedule, grid=(2, 3, 4), tokens=30)
    assert steps[0] is None and steps[1].tau == 1.25 and steps[2].tau == 1.5
    assert steps[1].order is steps[2].order
    assert torch.equal(steps[1].order, morton_order(2, 3, 4, tokens=30))
    assert not steps[1].applies_to(0) and steps[1].applies_to(1) and not steps[1].applies_to(47)
    dense = resolve_schedule("dense", "none", steps=2, label="s", stage=1)
    assert stage_steps(dense, grid=(1, 1, 1), tokens=1) == (None, None)
