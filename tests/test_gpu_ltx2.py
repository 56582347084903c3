"""Device LTX-2 video DiT against the CPU oracle on identical seeded inputs.

Full width (hidden 4096, 32 heads, so the QK RMSNorm spans all 4096 channels), short token grids
so the CPU oracle finishes in seconds. Seeds: weights S, latent S + 1, text S + 2 (N(0, 1)).
Positions: pixel-space patch bounds of the latent grid (scale 8/32/32, causal fix, 24 fps).
"""

from __future__ import annotations

import pytest
import torch

from oracle import ltx2 as ref
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer, precompute_freqs_cis
from kinomlx_b200.synthetic import ltx_weights, normal

pytestmark = pytest.mark.gpu


def _metrics(out, expect):
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return (float((o - e).norm() / e.norm()), float((o - e).abs().max() / e.abs().max()),
            float(torch.nn.functional.cosine_similarity(o, e, dim=0)))


def _positions(f, h, w):
    return ref.pixel_coords(ref.patch_grid_bounds(f, h, w))


def test_rope_tables_match_oracle():
    v = lcfg.BASELINE_VIDEO
    pos = _positions(3, 4, 8)
    c, s = precompute_freqs_cis(pos, v)
    rc, rs = ref.precompute_freqs_cis(pos, dim=v.dim, theta=v.theta, max_pos=v.max_pos, heads=v.heads)
    assert torch.equal(c, rc) and torch.equal(s, rs)


def test_one_block_velocity_matches_oracle(cuda_device):
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=0)
    grid = (3, 4, 8)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=1)
    context = normal((1, 64, v.context_dim), seed=2)
    pos = _positions(*grid)
    sigma = ref.DISTILLED_STAGE_1_SIGMAS[5]
    expect = ref.forward(w, latent, context, sigma, pos, v)
    model = LTXVideoTransformer(w, v, cuda_device)
    prepared = model.prepare(context, pos)
    out = model.run(prepared, latent.to(cuda_device), sigma).clone()
    rel_l2, max_rel, cos = _metrics(out, expect)
    assert rel_l2 <= 1e-2 and max_rel <= 2e-2 and cos >= 0.999, (rel_l2, max_rel, cos)


def test_denoise_tail_matches_oracle(cuda_device):
    """Two blocks over the last three distilled stage-1 steps with X0 + Euler fused into the
    final projection: final latent cosine >= 0.999."""
    v = lcfg.BASELINE_VIDEO.with_blocks(2)
    w = ltx_weights(v, seed=7)
    grid = (2, 6, 8)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=8)
    context = normal((1, 32, v.context_dim), seed=9)
    pos = _positions(*grid)
    sigmas = ref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = ref.denoise(w, latent, context, pos, sigmas, v)
    model = LTXVideoTransformer(w, v, cuda_device)
    out = ldn.denoise_video(model, latent, context, pos, sigmas)
    rel_l2, max_rel, cos = _metrics(out, expect)
    assert cos >= 0.999 and rel_l2 <= 3e-2, (rel_l2, max_rel, cos)


def test_config4_block_shapes_run(cuda_device):
    """BASELINE config 4 shapes for two blocks (9216 video tokens, 256 text tokens, width 4096),
    weights drawn on the GPU: finite, deterministic."""
    v = lcfg.BASELINE_VIDEO.with_blocks(2)
    w = ltx_weights(v, seed=3, device=cuda_device)
    model = LTXVideoTransformer(w, v, cuda_device)
    latent = normal((1, 16 * 18 * 32, v.in_channels), seed=4, device=cuda_device)
    context = normal((1, 256, v.context_dim), seed=5, device=cuda_device)
    prepared = model.prepare(context, _positions(16, 18, 32))
    a = model.run(prepared, latent, 0.725).clone()
    b = model.run(prepared, latent, 0.725).clone()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(a).all()) and torch.equal(a, b)
