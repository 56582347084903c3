"""Sol-Attn on the B200 (kino_sol_attention) against the CPU oracle restated from
kinomlx/models/ltx2/kernels/sol_attention.py and pinned in tests/test_sol_attention_oracle.py.

Routing compares mean-key scores with a limit; the device sums the block means and the scores in
another order than the oracle, so an entry whose score lies within float rounding of its limit
may route differently. The routes are therefore compared entry by entry, allowing a difference
only where the oracle's score is within 1e-4 (relative) of its limit, and the attention is
checked against the oracle's attention given the device's routes. Tolerances: the operands are
fp16 on both sides; the device keeps the probabilities in fp16 for the P V product (the oracle in
fp32), so the gate is 1e-2 relative L2 and 2e-2 max-normalised error."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import sol_attention as ref
from kinomlx_b200 import ops
from kinomlx_b200.kernels import sol_attention as sol
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu


def _inputs(tokens, heads, dtype, seed, scale=1.0):
    gen = torch.Generator().manual_seed(seed)
    mk = lambda: (torch.randn((tokens, heads * 128), generator=gen) * scale).to(dtype)
    q, k, v = mk(), mk(), mk()
    # a little shared structure so that routing is not uniform noise
    base = torch.randn((1, heads * 128), generator=gen)
    k = (k.float() + 0.5 * base).to(dtype)
    return q, k, v


def _oracle_routes(q, k, v, heads, order, tau):
    q16, k16, v16, qmean, kmean, vmean = ref.prepare(q, k, v, heads=heads, order=order.long())
    routes, _, _, _ = ref.route_blocks(qmean, kmean, tau=tau)
    # the margin of every entry: score - limit, relative
    h, nb, dim = qmean.shape
    keys = kmean.float()
    ls = dim ** -0.5 * ref.LOG2E
    scores = (qmean @ keys.transpose(1, 2)) * ls
    center = keys.mean(dim=1, keepdim=True)
    raw_mean = (qmean * center).sum(-1)
    var = ((keys - center) ** 2).mean(dim=1, keepdim=True)
    raw_var = (qmean ** 2 * var).sum(-1)
    limit = raw_mean * ls + tau * torch.sqrt(torch.clamp(raw_var, min=0) * ls * ls + ref.VARIANCE_EPSILON)
    margin = (scores - limit[..., None]).abs() / limit.abs().clamp(min=1e-3)[..., None]
    return (q16, k16, v16, kmean, vmean), routes, margin


CASES = [
    # tokens, heads, dtype, tau
    (1000, 2, torch.bfloat16, 0.5),      # partial last block (1000 = 15 x 64 + 40)
    (2048, 3, torch.float16, 1.0),
    (4096 + 64, 2, torch.bfloat16, 1.5),  # a CTA with a single query block
    (777, 4, torch.bfloat16, -0.25),
    (300, 2, torch.float16, 2.5),
]


@pytest.mark.parametrize("tokens,heads,dtype,tau", CASES)
def test_sol_attention_matches_oracle(cuda_device, tokens, heads, dtype, tau):
    q, k, v = _inputs(tokens, heads, dtype, seed=tokens + heads)
    order = sol.morton_order(1, 1, tokens) if tokens % 7 else torch.randperm(
        tokens, generator=torch.Generator().manual_seed(3)).to(torch.int32)
    dq, dk, dv = (x.to(cuda_device) for x in (q, k, v))
    got_routes = sol.routed_blocks(dq, dk, dv, heads=heads, tau=tau, order=order).cpu()
    got = sol.sol_attention(dq, dk, dv, heads=heads, tau=tau, order=order)
    torch.cuda.synchronize()
    ops.device_status()
    (q16, k16, v16, kmean, vmean), routes, margin = _oracle_routes(q, k, v, heads, order, tau)
    differ = got_routes != routes
    assert bool((margin[differ] < 1e-4).all()), f"{int(differ.sum())} routes differ away from the limit"
    assert int(differ.sum()) <= max(2, routes.numel() // 1000)
    routed = ref.attend(q16, k16, v16, kmean, vmean, got_routes)
    expect = torch.empty_like(routed)
    expect[order.long()] = routed
    m = metrics(got, expect.to(dtype))
    print(show(f"sol {tokens}x{heads} {dtype} tau {tau}", m), f"routed {float(routes.float().mean()):.3f}")
    assert got.dtype == dtype and m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("sol", m)


def test_every_block_routed_is_dense_attention(cuda_device):
    """tau far below every score: every block is routed, no centroid takes part, and the result
    is dense attention over the fp16 operands (the reference test's own property)."""
    tokens, heads = 1500, 2
    q, k, v = _inputs(tokens, heads, torch.bfloat16, seed=9)
    order = sol.morton_order(3, 20, 25)
    dq, dk, dv = (x.to(cuda_device) for x in (q, k, v))
    assert bool(sol.routed_blocks(dq, dk, dv, heads=heads, tau=-1e4, order=order).all())
    got = sol.sol_attention(dq, dk, dv, heads=heads, tau=-1e4, order=order)
    split = lambda x: x.half().float().reshape(tokens, heads, 128).transpose(0, 1)
    s = split(q) @ split(k).transpose(1, 2) / math.sqrt(128)
    dense = (torch.softmax(s, -1) @ split(v)).transpose(0, 1).reshape(tokens, -1)
    m = metrics(got, dense.to(torch.bfloat16))
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("all routed vs dense", m)


def test_gate_strided_inputs_and_config4_shape(cuda_device):
    """q, k, v as column views of one (tokens, 3 * width) projection (the LTX block's [v | q | k]
    buffer), a per-head gate, at config 4's 9216 tokens (16 x 18 x 32 Morton grid, 8 heads so
    the oracle stays quick)."""
    tokens, heads = 9216, 8
    width = heads * 128
    gen = torch.Generator().manual_seed(21)
    qkv = (torch.randn((tokens, 3 * width), generator=gen)).to(torch.bfloat16)
    gate = torch.rand((tokens, heads), generator=gen).to(torch.bfloat16)
    order = sol.morton_order(16, 18, 32)
    dev = qkv.to(cuda_device)
    vv, q, k = dev[:, :width], dev[:, width : 2 * width], dev[:, 2 * width :]
    routes = sol.routed_blocks(q, k, vv, heads=heads, tau=1.0, order=order).cpu()
    out = ops.sol_attention(q, k, vv, heads=heads, tau=1.0, order=order.to(cuda_device),
                            gate=gate.to(cuda_device))
    torch.cuda.synchronize()
    cq, ck, cv = qkv[:, width : 2 * width], qkv[:, 2 * width :], qkv[:, :width]
    q16, k16, v16, _, kmean, vmean = ref.prepare(cq, ck, cv, heads=heads, order=order.long())
    routed = ref.attend(q16, k16, v16, kmean, vmean, routes)
    expect = torch.empty_like(routed)
    expect[order.long()] = routed
    expect = (expect.to(torch.bfloat16).reshape(tokens, heads, 128).float() * gate.float()[..., None])
    m = metrics(out, expect.reshape(tokens, width).to(torch.bfloat16))
    print(show("sol 9216 x 8 gated", m), f"routed {float(routes.float().mean()):.3f}")
    assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show("gated", m)


def test_out_of_range_order_is_reported_not_read(cuda_device):
    """An order that is not a permutation (one index past the rows) is caught by the kernels'
    own bounds checks: no read or write past the tensors, an error from the status call."""
    tokens, heads = 256, 2
    q, k, v = (x.to(cuda_device) for x in _inputs(tokens, heads, torch.bfloat16, seed=5))
    order = torch.arange(tokens, dtype=torch.int32)
    order[17] = tokens
    ops.sol_attention(q, k, v, heads=heads, tau=1.0, order=order.to(cuda_device))
    with pytest.raises(RuntimeError, match="out-of-range index"):
        ops.device_status()
    ops.device_status()  # cleared


def test_ltx_block_with_a_sparse_step(cuda_device):
    """The LTX-2 video block's self-attention through Sol-Attn: every layer dense by the step's
    dense layers is the dense forward bit for bit; every block routed is the dense forward up to
    the fp16 operands; a real tau runs and stays close to dense."""
    from oracle import ltx2 as lref
    from kinomlx_b200.ltx2 import config as lcfg
    from kinomlx_b200.ltx2.sparse_attention import SparseAttentionStep
    from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
    from kinomlx_b200.synthetic import ltx_weights, normal

    v = lcfg.BASELINE_VIDEO.with_blocks(2)
    w = ltx_weights(v, seed=81)
    grid = (4, 6, 8)
    tokens = grid[0] * grid[1] * grid[2]
    latent = normal((1, tokens, v.in_channels), seed=82).to(cuda_device)
    context = normal((1, 32, v.context_dim), seed=83).to(cuda_device)
    pos = lref.pixel_coords(lref.patch_grid_bounds(*grid))
    model = LTXVideoTransformer(w, v, cuda_device)
    prep = model.prepare(context, pos)
    dense = model.run(prep, latent, 0.725).clone()
    order = sol.morton_order(*grid)
    off = SparseAttentionStep(1.0, frozenset({0, 1}), order)
    assert torch.equal(model.run(prep, latent, 0.725, sparse=off), dense)
    every = SparseAttentionStep(-1e4, frozenset(), order)
    m = metrics(model.run(prep, latent, 0.725, sparse=every), dense)
    assert m["rel_l2"] <= 1e-2 and m["cos"] >= 0.9999, show("all routed vs dense", m)
    real = SparseAttentionStep(1.0, frozenset({0}), order)
    a = model.run(prep, latent, 0.725, sparse=real).clone()
    b = model.run(prep, latent, 0.725, sparse=real).clone()
    assert torch.equal(a, b) and bool(torch.isfinite(a).all())
    print(show("tau 1 (layer 0 dense) vs dense", metrics(a, dense)))
