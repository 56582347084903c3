"""The B200 neighborhood attention (kino_neighborhood_attention) against the CPU oracle restated
from kinomlx/models/ltx2/kernels/neighborhood_attention.py and pinned in
tests/test_neighborhood_attention_oracle.py: the reference test's grids (tails on every axis,
batches, heads, query scales), windows beyond the reference kernels' contract, the exact
properties of the smallest and largest windows, and the decoder's final-stage shape checked on a
sample of queries. The device keeps the probabilities in fp16 for the P V product (the oracle in
fp32), so the gates are 1e-2 relative L2 and 2e-2 max-normalised error."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import neighborhood_attention as ref
from kinomlx_b200 import ops
from kinomlx_b200.kernels import neighborhood_attention as na
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu

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


def _inputs(batch, grid, heads, seed, q_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    shape = (batch, *grid, heads, 64)
    q = (torch.randn(shape, generator=g) * 0.125 * q_scale).half()
    return q, torch.randn(shape, generator=g).half(), torch.randn(shape, generator=g).half()


@pytest.mark.parametrize(("batch", "grid", "heads", "window", "q_scale"), CASES)
def test_reference_grids_match_oracle(cuda_device, batch, grid, heads, window, q_scale):
    q, k, v = _inputs(batch, grid, heads, sum(grid) + heads, q_scale)
    dq, dk, dv = (x.to(cuda_device) for x in (q, k, v))
    assert na.applies(dq, dk, dv, window=window)
    got = na.neighborhood_attention(dq, dk, dv, window=window)
    torch.cuda.synchronize()
    ops.device_status()
    expect = ref.neighborhood_attention(q, k, v, window=window)
    m = metrics(got, expect)
    print(show(f"NA {batch}x{grid}x{heads} window {window} scale {q_scale}", m))
    assert got.dtype == torch.float16 and got.shape == q.shape
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("neighborhood", m)


@pytest.mark.parametrize(("grid", "window"), [((5, 6, 40), (5, 5, 5)), ((3, 17, 9), (1, 9, 3)),
                                              ((9, 7, 70), (3, 3, 33))])
def test_windows_beyond_the_reference_kernels(cuda_device, grid, window):
    """Windows and grids the reference's kernels leave to its masked path (a 33-wide window
    spans two key boxes along W, grids narrower than a box on H or W)."""
    assert not ref.supports((1, *grid, 2, 64), window)
    q, k, v = _inputs(1, grid, 2, 7)
    got = ops.neighborhood_attention(*(x.to(cuda_device) for x in (q, k, v)), window=window)
    expect = ref.neighborhood_attention(q, k, v, window=window)
    m = metrics(got, expect)
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show(f"window {window}", m)


def test_unit_window_is_the_values_and_whole_grid_window_is_dense(cuda_device):
    q, k, v = _inputs(2, (3, 5, 7), 3, 11)
    dq, dk, dv = (x.to(cuda_device) for x in (q, k, v))
    assert torch.equal(ops.neighborhood_attention(dq, dk, dv, window=(1, 1, 1)).cpu(), v)
    got = ops.neighborhood_attention(dq, dk, dv, window=(3, 5, 7))
    flat = lambda x: x.reshape(2, -1, 3, 64).float().transpose(1, 2)
    dense = (torch.softmax(flat(q) @ flat(k).transpose(-1, -2), -1) @ flat(v)).transpose(1, 2)
    m = metrics(got, dense.reshape(q.shape).half())
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("whole-grid window vs dense", m)


def test_decoder_final_stage_shape_on_sampled_queries(cuda_device):
    """The decoder's final-stage call (121 x 112 x 192 queries, four heads, 11 x 11 x 11), the
    one the reference times: every query on the device, 4096 sampled queries (edges and
    corners included) against their windows on the CPU."""
    grid, heads, window = (121, 112, 192), 4, (11, 11, 11)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    shape = (1, *grid, heads, 64)
    dq = (torch.randn(shape, generator=g, device=cuda_device) * 0.125).half()
    dk = torch.randn(shape, generator=g, device=cuda_device).half()
    dv = torch.randn(shape, generator=g, device=cuda_device).half()
    assert na.applies(dq, dk, dv, window=window)
    got = na.neighborhood_attention(dq, dk, dv, window=window)
    torch.cuda.synchronize()
    ops.device_status()
    tokens = math.prod(grid)
    pick = torch.cat([torch.randint(0, tokens, (4000,), generator=torch.Generator().manual_seed(6)),
                      torch.tensor([0, tokens - 1, grid[2] - 1, tokens - grid[2]])])
    pick = torch.cat([pick, torch.arange(0, tokens, tokens // 92)[:92]])
    keys = ref.window_keys(grid, window)[pick]  # (n, 1331)
    qf = dq.reshape(tokens, heads, 64)[pick.to(cuda_device)].float().cpu()
    kh = dk.reshape(tokens, heads, 64).cpu()
    vh = dv.reshape(tokens, heads, 64).cpu()
    parts = []
    for start in range(0, pick.numel(), 256):  # the sampled queries' windows, 256 at a time
        sel = keys[start : start + 256]
        scores = torch.einsum("nhd,nkhd->nhk", qf[start : start + 256], kh[sel].float())
        parts.append(torch.einsum("nhk,nkhd->nhd", torch.softmax(scores, -1), vh[sel].float()))
    expect = torch.cat(parts).half()
    m = metrics(got.reshape(tokens, heads, 64)[pick.to(cuda_device)], expect)
    print(show("final stage, sampled queries", m))
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("final stage", m)
