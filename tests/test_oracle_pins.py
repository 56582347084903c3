"""The CPU oracle against the known answers the reference's own tests hold for this path.

Each test names the reference test it restates. These pin the restatement; nothing here needs a
GPU.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import flux2, fused_ops, ltx2, video_vae


@pytest.mark.parametrize(
    ("tokens", "steps", "midpoint"),
    [
        (1024, 4, 0.8839818317017591),
        (4096, 4, 0.908143922521333),
        (4300, 10, 0.9067067588045681),
        (4301, 10, 0.7657912730789151),
        (4096, 200, 0.7595102922715895),
        (16384, 4, 0.9619472529114758),
    ],
)
def test_klein_schedule_midpoints(tokens, steps, midpoint):
    """tests/models/flux2/test_sampling.py:214-227 (BFL empirical mu and shift)."""
    assert flux2.schedule(tokens, steps)[steps // 2].item() == pytest.approx(midpoint, abs=1e-7)


def test_schedule_endpoints_and_euler_rounding_order():
    """tests/models/flux2/test_sampling.py:200-211."""
    sigmas = flux2.schedule(384, 4)
    assert sigmas[0].item() == 1 and sigmas[-1].item() == 0
    assert bool((sigmas[1:] < sigmas[:-1]).all())
    source = torch.tensor([0.5], dtype=torch.bfloat16)
    velocity = torch.tensor([1.25], dtype=torch.bfloat16)
    actual = flux2.euler_step(source, velocity, torch.tensor(-0.123, dtype=torch.float32))
    increment = torch.tensor(-0.123, dtype=torch.bfloat16) * velocity
    assert torch.equal(actual, (source.float() + increment.float()).to(torch.bfloat16))


def test_double_precision_rope_grid_matches_float64():
    """tests/models/ltx2/transformer/test_primitives.py:115-133."""
    positions = torch.tensor([[[[0.0, 1.0]]]])
    cos, sin = ltx2.precompute_freqs_cis(positions, dim=8, theta=10000.0, max_pos=(20,), heads=2)
    grid = np.power(10000.0, np.linspace(0.0, 1.0, 4, dtype=np.float64))
    angles = (grid * np.pi / 2).astype(np.float32) * np.float32(2 * 0.5 / 20 - 1)
    exp_cos = torch.from_numpy(np.cos(angles).astype(np.float32)).reshape(1, 2, 1, 2)
    exp_sin = torch.from_numpy(np.sin(angles).astype(np.float32)).reshape(1, 2, 1, 2)
    assert torch.allclose(cos, exp_cos, atol=1e-6)
    assert torch.allclose(sin, exp_sin, atol=1e-6)


def test_ltx_distilled_sigma_pins():
    """kinomlx/models/ltx2/sigmas.py:24-52: literal schedules rounded to fp32."""
    expect = [1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0]
    got = ltx2.DISTILLED_STAGE_1_SIGMAS
    assert len(got) == 9
    for a, b in zip(got, expect):
        assert a == float(np.float32(b))
    assert ltx2.DISTILLED_STAGE_2_SIGMAS == got[5:]


def test_trapezoid_mask_and_tile_intervals():
    """tests/models/ltx2/video_vae/test_tiling.py:441-446, 574-596."""
    mask = video_vae.compute_trapezoidal_mask_1d(5, 2, 2)
    assert torch.allclose(mask, torch.tensor([1 / 3, 2 / 3, 1.0, 2 / 3, 1 / 3]))
    assert [e - s for s, e in video_vae.tile_intervals(361, 104, 92, 6)] == [104, 104, 104, 85]
    assert video_vae.tile_intervals(10, 16, 8, 6) == [(0, 10)]
    assert video_vae.tile_intervals(361, 64, 52, 6)[:6] == [
        (0, 64), (52, 116), (104, 168), (156, 220), (208, 272), (260, 324)
    ]
    assert video_vae.tile_intervals(61, 40, 28, 6) == [(0, 40), (28, 61)]


def test_split_axis_config5_tiles():
    """BASELINE config 5 tiling (8-latent tiles, 2-latent overlap over an 18 x 32 latent):
    3 x 5 = 15 tiles with 2-latent ramps between neighbours (tiling.py:834-863)."""
    th = video_vae.split_axis(18, 8, 2)
    tw = video_vae.split_axis(32, 8, 2)
    assert list(zip(th.starts, th.ends)) == [(0, 8), (6, 14), (12, 18)]
    assert list(zip(tw.starts, tw.ends)) == [(0, 8), (6, 14), (12, 20), (18, 26), (24, 32)]
    assert th.left_ramps == [0, 2, 2] and th.right_ramps == [2, 2, 0]
    for length, tile, overlap in [(37, 8, 2), (9, 8, 3), (100, 16, 5)]:
        t = video_vae.split_axis(length, tile, overlap)
        assert all(e - s <= tile for s, e in zip(t.starts, t.ends))
        assert t.starts[0] == 0 and t.ends[-1] == length


def test_gelu_silu_bounds_against_fp32():
    """tests/kernels/test_fused_ops.py: bf16 GELU max-abs 4e-6 and SiLU exact against the fp32
    formula rounded once, on linspace(-8, 8, 65536)."""
    x = torch.linspace(-8, 8, 65536).to(torch.bfloat16)
    f = x.float()
    gelu = (0.5 * f * (1 + torch.tanh(0.7978845608028654 * (f + 0.044715 * f**3)))).to(torch.bfloat16)
    silu = (f / (1 + torch.exp(-f))).to(torch.bfloat16)
    assert float((fused_ops.gelu_approx(x).float() - gelu.float()).abs().max()) <= 4e-6
    assert torch.equal(fused_ops.silu(x), silu)


def test_split_rope_matches_reference_graph_on_self_test_recipe():
    """kinomlx/kernels/split_rope.py:87-98, 120-136: the oracle rotation equals the reference
    graph's formula (one fp32 rounding per product) on the kernel's self-test inputs."""
    batch, heads, tokens, half = 2, 3, 7, 5
    count = batch * tokens * heads * 2 * half
    value = (torch.sin(torch.arange(count, dtype=torch.float32) * 0.7310585) * 3.0).to(torch.bfloat16)
    value = value.reshape(batch, tokens, heads * 2 * half)
    angles = torch.arange(tokens * heads * half, dtype=torch.float32) * 0.4142135
    angles = angles.reshape(1, tokens, heads, half).transpose(1, 2)
    cos, sin = torch.cos(angles), torch.sin(angles)
    hf = value.reshape(batch, tokens, heads, 2 * half).transpose(1, 2).float()
    first, second = hf[..., :half], hf[..., half:]
    graph = torch.cat([first * cos - second * sin, first * sin + second * cos], -1)
    graph = graph.transpose(1, 2).reshape(value.shape).to(torch.bfloat16)
    assert torch.equal(ltx2.apply_split_rotary_emb(value, cos, sin), graph)


def test_pixel_norm_is_stepwise():
    """kinomlx/kernels/fused_ops.py:460-476: square, mean, + eps, sqrt, divide, each rounded."""
    x = (torch.randn(4, 6, 64, generator=torch.Generator().manual_seed(3)) * 3).to(torch.bfloat16)
    sq = x * x
    rms = torch.sqrt(sq.float().mean(-1, keepdim=True).to(torch.bfloat16) + 1e-8)
    assert torch.equal(fused_ops.pixel_norm(x, eps=1e-8), x / rms)


def test_timestep_features_match_formula():
    t = torch.tensor([500.0])
    f = ltx2.timestep_features(t)
    freq = torch.exp(-math.log(10000) * torch.arange(128, dtype=torch.float32) / 128)
    assert torch.allclose(f, torch.cat([torch.cos(500 * freq), torch.sin(500 * freq)])[None])
