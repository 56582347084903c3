"""Pins of the Sol-Attn oracle (oracle/sol_attention.py) against the reference's own tests
(tests/models/ltx2/test_sol_attention.py of KinoMLX): Morton order against an independent bit
interleave, block cubes, appended tokens, the large-tau routing's known answers, routing every
block equals dense attention, the oracle against the reference test's closed-form fp32 formula,
preparation, saturation and refusals. CPU only."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import sol_attention as sol

HEADS = 2
GRID = (4, 8, 12)  # 384 grid tokens plus 33 appended: seven blocks, the last one partial
TOKENS = 417


def _python_morton(frames: int, height: int, width: int) -> list[int]:
    bits = max(frames, height, width).bit_length()

    def spread(value: int) -> int:
        code = 0
        for bit in range(bits):
            code |= ((value >> bit) & 1) << (3 * bit)
        return code

    codes = [spread(f) | spread(h) << 1 | spread(w) << 2
             for f in range(frames) for h in range(height) for w in range(width)]
    return sorted(range(len(codes)), key=codes.__getitem__)


@pytest.mark.parametrize("grid", [(5, 3, 7), (4, 4, 4), (1, 6, 9), (16, 14, 24)])
def test_morton_order_matches_an_independent_interleave(grid):
    assert sol.morton_order(*grid).tolist() == _python_morton(*grid)


def test_morton_blocks_are_cubes_and_appended_tokens_follow():
    first = sol.morton_order(8, 8, 8)[:64].tolist()
    cells = {(i // 64, (i // 8) % 8, i % 8) for i in first}
    assert cells == {(f, h, w) for f in range(4) for h in range(4) for w in range(4)}
    order = sol.morton_order(2, 3, 4, tokens=30)
    assert sorted(order[:24].tolist()) == list(range(24))
    assert order[24:].tolist() == list(range(24, 30))
    with pytest.raises(ValueError, match="cannot hold"):
        sol.morton_order(2, 3, 4, tokens=23)


def _inputs(dtype: torch.dtype, seed: int):
    """The reference test's scenario: a smooth shared component gives blocks distinct means, small
    queries flatten the softmax so unrouted blocks carry a real share of the output."""
    g = torch.Generator().manual_seed(seed)
    phase = torch.arange(TOKENS, dtype=torch.float32)[:, None] * 0.05
    cols = torch.arange(HEADS * sol.HEAD_DIM, dtype=torch.float32)[None, :]
    shared = 2.0 * torch.sin(phase + cols * 0.3)
    r = lambda: torch.randn((TOKENS, HEADS * sol.HEAD_DIM), generator=g)
    q = 0.15 * (r() + shared)
    k = r() + shared
    v = r()
    return q.to(dtype), k.to(dtype), v.to(dtype)


def _rel(actual: torch.Tensor, expected: torch.Tensor) -> float:
    d = actual.float() - expected.float()
    return float(torch.sqrt((d * d).sum() / (expected.float() ** 2).sum()))


def _closed_form(q, k, v, routes, kmean, vmean):
    """The reference test's fp32 Sol-Attn of routing-order inputs on a given routing (natural
    exponent, proxies weighted by block length)."""
    tokens = q.shape[0]
    blocks = sol.block_count(tokens)
    lengths = torch.clamp(tokens - torch.arange(blocks) * sol.BLOCK, max=sol.BLOCK).float()
    tb = torch.arange(tokens) // sol.BLOCK
    scale = sol.HEAD_DIM ** -0.5
    outs = []
    for h in range(HEADS):
        cols = slice(h * sol.HEAD_DIM, (h + 1) * sol.HEAD_DIM)
        qh, kh, vh = (x[:, cols].float() for x in (q, k, v))
        rows = routes[h].float()[tb]
        scores = (qh @ kh.T) * scale
        peak = scores.max(-1, keepdim=True).values
        exact = torch.exp(scores - peak) * rows[:, tb]
        proxy = torch.exp((qh @ kmean[h].float().T) * scale - peak) * (1.0 - rows) * lengths
        num = exact @ vh + proxy @ vmean[h].float()
        outs.append(num / (exact.sum(-1) + proxy.sum(-1))[:, None])
    return torch.cat(outs, -1)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("tau", [-1.0, 0.5, 1.0, 1.5])
def test_oracle_matches_the_closed_form_on_its_own_routing(dtype, tau):
    q, k, v = _inputs(dtype, 11)
    order = sol.morton_order(*GRID, tokens=TOKENS)
    out = sol.sol_attention(q, k, v, heads=HEADS, tau=tau, order=order)
    gq, gk, gv, qmean, kmean, vmean = sol.prepare(q, k, v, heads=HEADS, order=order)
    routes, _, counts, _ = sol.route_blocks(qmean, kmean, tau=tau)
    expected = _closed_form(gq, gk, gv, routes, kmean, vmean)[torch.argsort(order)]
    assert out.dtype == dtype and out.shape == q.shape
    assert _rel(out, expected) < {torch.float16: 1e-3, torch.bfloat16: 6e-3}[dtype]
    assert int(counts.min()) >= 2  # neighbours always route
    if tau >= 0.5:
        assert int(counts.max()) < sol.block_count(TOKENS)  # and some blocks are left out


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_routing_every_block_is_dense_attention(dtype):
    q, k, v = _inputs(dtype, 12)
    order = sol.morton_order(*GRID, tokens=TOKENS)
    out = sol.sol_attention(q, k, v, heads=HEADS, tau=-1e6, order=order)
    sh = lambda x: x.float().reshape(TOKENS, HEADS, sol.HEAD_DIM).transpose(0, 1)
    att = torch.softmax(sh(q) @ sh(k).transpose(1, 2) * sol.HEAD_DIM ** -0.5, -1) @ sh(v)
    dense = att.transpose(0, 1).reshape(TOKENS, HEADS * sol.HEAD_DIM)
    assert _rel(out, dense) < {torch.float16: 1e-3, torch.bfloat16: 6e-3}[dtype]


def test_a_large_tau_routes_only_each_block_and_its_neighbours():
    q, k, v = _inputs(torch.float16, 13)
    order = sol.morton_order(*GRID, tokens=TOKENS)
    *_, qmean, kmean, _ = sol.prepare(q, k, v, heads=HEADS, order=order)
    routes, lists, counts, bits = sol.route_blocks(qmean, kmean, tau=1e6)
    blocks = sol.block_count(TOKENS)
    index = torch.arange(blocks)
    band = (index[:, None] - index[None, :]).abs() <= 1
    assert torch.equal(routes, band.expand_as(routes))
    assert counts[0].tolist() == [2] + [3] * (blocks - 2) + [2]
    assert lists[0, 3, :3].tolist() == [2, 3, 4]
    assert int(bits[0, 3, 0]) == 0b11100


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_preparation_gathers_converts_and_averages(dtype):
    q, k, v = _inputs(dtype, 14)
    order = sol.morton_order(*GRID, tokens=TOKENS)
    gq, _, gv, qmean, _, vmean = sol.prepare(q, k, v, heads=HEADS, order=order)
    assert gq.dtype == torch.float16 and vmean.dtype == torch.float16
    assert torch.equal(gq, q[order].half()) and torch.equal(gv, v[order].half())
    blocks = sol.block_count(TOKENS)
    padded = torch.nn.functional.pad(q[order].float(), (0, 0, 0, blocks * sol.BLOCK - TOKENS))
    lengths = torch.clamp(TOKENS - torch.arange(blocks) * sol.BLOCK, max=sol.BLOCK).float()
    sums = padded.reshape(blocks, sol.BLOCK, HEADS, sol.HEAD_DIM).sum(1)
    expected = (sums / lengths[:, None, None]).transpose(0, 1)
    assert torch.allclose(qmean, expected, rtol=1e-5, atol=1e-6)


def test_bfloat16_values_beyond_float16_saturate():
    q, k, v = _inputs(torch.bfloat16, 15)
    v = torch.cat([torch.full((1, v.shape[1]), 1e5, dtype=torch.bfloat16), v[1:]])
    order = sol.morton_order(*GRID, tokens=TOKENS)
    assert bool(torch.isfinite(sol.sol_attention(q, k, v, heads=HEADS, tau=1.0, order=order)).all())


def test_inputs_outside_the_contract_are_refused():
    q, k, v = _inputs(torch.float16, 16)
    order = sol.morton_order(*GRID, tokens=TOKENS)
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        sol.sol_attention(q.float(), k.float(), v.float(), heads=HEADS, tau=1.0, order=order)
    with pytest.raises(ValueError, match="4 \\* 128"):
        sol.sol_attention(q, k, v, heads=4, tau=1.0, order=order)
    with pytest.raises(ValueError, match="one index per token"):
        sol.sol_attention(q, k, v, heads=HEADS, tau=1.0, order=order[:-1])
    with pytest.raises(ValueError, match="finite"):
        sol.sol_attention(q, k, v, heads=HEADS, tau=math.inf, order=order)
