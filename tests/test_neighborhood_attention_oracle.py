"""Pins of the neighborhood-attention oracle (oracle/neighborhood_attention.py) against the
reference's own tests (tests/models/ltx2/test_neighborhood_attention.py of KinoMLX): the window
formula against an independent masked dense attention on the reference test's grids (tails on
every axis, batches, heads, query scales), values outside a window never reaching its query,
and every shape/window/size refusal of the host contract. CPU only."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import neighborhood_attention as na

CASES = [  # (batch, grid, heads, window, q_scale): the reference test's parametrisation
    (1, (19, 13, 15), 2, (11, 11, 11), 1.0),
    (2, (18, 12, 12), 3, (11, 11, 11), 1.0),
    (1, (20, 14, 13), 2, (11, 11, 11), 8.0),
    (1, (14, 14, 16), 2, (11, 11, 11), 1.0),
    (1, (4, 9, 16), 3, (3, 7, 7), 1.0),
    (2, (7, 11, 21), 2, (3, 7, 7), 4.0),
    (1, (3, 8, 16), 2, (3, 5, 5), 1.0),
    (1, (6, 9, 19), 4, (3, 5, 5), 1.0),
]


def _inputs(batch, grid, heads, seed, q_scale):
    """Scaled queries (the decoder scales them by D^-0.5 before the call), fp16."""
    g = torch.Generator().manual_seed(seed)
    shape = (batch, *grid, heads, na.HEAD_DIM)
    q = (torch.randn(shape, generator=g) * 0.125 * q_scale).half()
    return q, torch.randn(shape, generator=g).half(), torch.randn(shape, generator=g).half()


def _masked_dense(q, k, v, window):
    """Independent restatement: dense fp32 attention with every key outside the query's
    per-axis window interval masked."""
    batch, gt, gh, gw, heads, dim = q.shape
    coords = torch.stack(torch.meshgrid(torch.arange(gt), torch.arange(gh), torch.arange(gw),
                                        indexing="ij"), -1).reshape(-1, 3)
    allowed = torch.ones(coords.shape[0], coords.shape[0], dtype=torch.bool)
    for axis, (length, size) in enumerate(zip((gt, gh, gw), window)):
        lo = [max(0, min(i - size // 2, length - size)) for i in range(length)]
        start = torch.tensor(lo)[coords[:, axis]]
        pos = coords[:, axis]
        allowed &= (pos[None, :] >= start[:, None]) & (pos[None, :] < start[:, None] + size)
    flat = lambda x: x.reshape(batch, -1, heads, dim).float().transpose(1, 2)
    scores = flat(q) @ flat(k).transpose(-1, -2)
    out = torch.softmax(scores.masked_fill(~allowed, -math.inf), -1) @ flat(v)
    return out.transpose(1, 2).reshape(q.shape)


@pytest.mark.parametrize(("batch", "grid", "heads", "window", "q_scale"), CASES)
def test_window_formula_matches_masked_dense_attention(batch, grid, heads, window, q_scale):
    q, k, v = _inputs(batch, grid, heads, sum(grid) + heads, q_scale)
    assert na.applies(q.shape, k.shape, v.shape, (q.dtype, k.dtype, v.dtype), window=window)
    out = na.neighborhood_attention(q, k, v, window=window)
    expect = _masked_dense(q, k, v, window)
    assert out.shape == q.shape and out.dtype == torch.float16
    assert bool(torch.isfinite(out).all())
    diff = out.float() - expect
    assert float(torch.sqrt((diff * diff).sum() / (expect * expect).sum())) < 1e-3


def test_windows_shift_inward_and_keep_their_size():
    assert na.window_starts(7, 3).tolist() == [0, 0, 1, 2, 3, 4, 4]
    assert na.window_starts(11, 11).tolist() == [0] * 11
    keys = na.window_keys((5, 4, 6), (3, 3, 5))
    assert keys.shape == (5 * 4 * 6, 45)
    assert all(len(set(row)) == 45 for row in keys.tolist())


def test_values_outside_a_window_do_not_reach_its_query():
    """Query (0, 0, 0)'s window spans frames 0-10 of 18: large values from frame 11 on leave its
    output bit for bit and reach the last frame's queries."""
    grid, window = (18, 12, 12), (11, 11, 11)
    q, k, v = _inputs(1, grid, 2, 5, 1.0)
    spiked = v.clone()
    spiked[:, 11:] += 1000.0
    plain = na.neighborhood_attention(q, k, v, window=window)
    other = na.neighborhood_attention(q, k, spiked, window=window)
    assert torch.equal(other[0, 0, 0, 0], plain[0, 0, 0, 0])
    assert not torch.equal(other[0, -1, 0, 0], plain[0, -1, 0, 0])


@pytest.mark.parametrize("window", [(11, 11, 11), (3, 7, 7)])
def test_applies_refuses_what_the_kernels_do_not_compute(window):
    shape, h = (1, 19, 13, 16, 2, 64), torch.float16
    assert na.applies(shape, shape, shape, (h, h, h), window=window)
    assert not na.applies(shape, shape, shape, (torch.bfloat16,) * 3, window=window)
    short = (1, 19, 13, 15, 2, 64)
    assert not na.applies(shape, short, shape, (h, h, h), window=window)
    assert not na.applies(shape, shape, shape, (h, h, h), window=(window[0], window[1], 4))
    assert not na.applies(shape, shape, shape, (h, h, h), window=(window[0], window[1], 17))
    wide = (1, 19, 13, 16, 2, 128)
    assert not na.applies(wide, wide, wide, (h, h, h), window=window)
    small = (1, 2, 13, 16, 2, 64)
    assert not na.applies(small, small, small, (h, h, h), window=window)
    huge = (1, 1024, 1024, 64, 2, 64)  # past 2**31 elements: still taken
    assert na.applies(huge, huge, huge, (h, h, h), window=window)
    assert na.launch_fits((1024, 1024, 64), window)
    assert not na.launch_fits((65_536, 2048, 2048), window)
    vast = (1, 65_536, 2048, 2048, 2, 64)
    assert not na.applies(vast, vast, vast, (h, h, h), window=window)
