"""LTX-2.5 diffusion video decoder, host side (no GPU): the oracle against the reference's own
known answers (tests/models/ltx2/video_vae/test_diffusion_decoder.py: the patchify round trip,
the minimum latent grid and the decoded shapes of its miniature decoder), the configuration's
checks (kinomlx/models/ltx2/video_vae/config.py:213-257) and the host-made RoPE tables."""

from __future__ import annotations

import pytest
import torch

from oracle import diffusion_decoder as dref
from kinomlx_b200.ltx2.diffusion_decoder import DiffusionDecoderConfig, rope_split, rope_tables
from kinomlx_b200.synthetic import diffusion_decoder_weights, normal


def mini_config(**changes) -> DiffusionDecoderConfig:
    """The reference test's miniature decoder (test_diffusion_decoder.py:40-56)."""
    fields = dict(head_dim=8, stage_channels=(64, 32, 16, 16, 8), stage_depths=(1, 1, 1, 1, 1),
                  stage_kernels=((3, 3, 3),) * 4,
                  upsample_strides=((1, 2, 2), (2, 1, 1), (2, 2, 2), (2, 2, 2)),
                  upsample_channel_reductions=(2, 2, 1, 2), stage5_kernel=(3, 3, 3), patch_size=2,
                  t_emb_dim=32, spatial_compression_ratio=16, temporal_compression_ratio=8,
                  latent_channels=8)
    fields.update(changes)
    return DiffusionDecoderConfig(**fields)


def test_patchify_round_trip_preserves_ltx_packing():
    source = torch.arange(1 * 2 * 3 * 4 * 6, dtype=torch.float32).reshape(1, 2, 3, 4, 6)
    packed = dref.patchify_spatial(source, 2)
    assert tuple(packed.shape) == (1, 8, 3, 2, 3)
    assert torch.equal(dref.unpatchify_spatial(packed, 2), source)
    # packed channel c * p * p + pw * p + ph holds pixel (h * p + ph, w * p + pw)
    c, pw, ph, f, h, w = 1, 1, 0, 2, 1, 2
    assert packed[0, c * 4 + pw * 2 + ph, f, h, w] == source[0, c, f, h * 2 + ph, w * 2 + pw]


def test_config_checks_follow_the_reference():
    with pytest.raises(ValueError, match="stage_channels"):
        mini_config(upsample_channel_reductions=(2, 2, 2, 2))
    with pytest.raises(ValueError, match="divide by head_dim"):
        mini_config(head_dim=16)
    with pytest.raises(ValueError, match="temporal stride"):
        mini_config(temporal_compression_ratio=4)
    with pytest.raises(ValueError, match="spatial stride"):
        mini_config(spatial_compression_ratio=32)
    with pytest.raises(ValueError, match="odd"):
        mini_config(stage5_kernel=(3, 4, 3))
    with pytest.raises(ValueError, match="model_output_type"):
        mini_config(model_output_type="eps")


@pytest.mark.parametrize("latent_shape, expect", [((1, 8, 2, 3, 3), (1, 3, 9, 48, 48)),
                                                  ((1, 8, 2, 1, 1), (1, 3, 9, 16, 16))])
def test_oracle_decodes_the_reference_shapes(latent_shape, expect):
    """test_full_decoder_is_seeded_and_single_covering_tile_is_exact and
    test_short_and_narrow_latent_is_padded_internally_then_cropped: the minimum grid (3, 3, 3)
    and the cropped output shapes; x_t of the configuration's working shape."""
    cfg = mini_config()
    assert cfg.minimum_latent_shape() == dref.minimum_latent_shape(cfg) == (3, 3, 3)
    w = diffusion_decoder_weights(cfg, seed=3)
    latent = normal(latent_shape, seed=4, dtype=torch.float32)
    noise = normal(cfg.working_pixel_shape(latent_shape), seed=5)
    assert cfg.working_pixel_shape(latent_shape) == dref.working_pixel_shape(latent_shape, cfg)
    out = dref.decode(latent, noise, w, cfg)
    assert tuple(out.shape) == expect
    assert torch.isfinite(out.float()).all()


def test_rope_tables_and_sections():
    assert rope_split(64) == dref.rope_split(64) == (16, 24, 24)
    assert rope_split(8) == (0, 4, 4)  # the miniature decoder's: 2 + 3 + 3 is odd, no t section
    grid = (5, 7, 9)
    host = rope_tables(64, grid)
    assert torch.equal(host, torch.cat([t.reshape(-1) for t in dref.rope_tables(64, grid)]))
    # frame 3's first pair turns by 3 radians, row 0 not at all
    assert host[3 * 8].item() == pytest.approx(torch.cos(torch.tensor(3.0)).item())
    assert host[2 * 5 * 8 : 2 * 5 * 8 + 12].eq(1.0).all()


def test_rope3d_rotates_each_section_by_its_axis():
    """A vector of ones rotated at (t, h, w) = (2, 0, 0): only the t section's pairs move."""
    x = torch.ones((1, 3, 2, 2, 1, 64), dtype=torch.float32)
    y = dref.rope3d(x, 64)
    assert torch.equal(y[0, 0, 0, 0], x[0, 0, 0, 0])
    assert not torch.equal(y[0, 0, 1, 1, 0, 16:], x[0, 0, 1, 1, 0, 16:])
    assert not torch.equal(y[0, 2, 0, 0, 0, :16], x[0, 2, 0, 0, 0, :16])
    assert torch.equal(y[0, 2, 0, 0, 0, 16:], x[0, 2, 0, 0, 0, 16:])


def test_copy_dims_merge_and_order():
    """The strided copy's host-side dimension list (ops._copy_dims): contiguous runs merge on
    both sides, size-1 dimensions vanish, broadcasts keep a zero source stride, and applying the
    list element by element reproduces the permuted copy."""
    from kinomlx_b200.ops import _copy_dims

    x = torch.arange(2 * 3 * 4 * 5).reshape(2, 3, 4, 5)
    assert _copy_dims(x.shape, x.stride(), x.stride()) == [[120, 1, 1]]
    p = x.permute(0, 2, 1, 3)  # (2, 4, 3, 5) view
    out = torch.empty(p.shape, dtype=x.dtype)
    dims = _copy_dims(p.shape, p.stride(), out.stride())
    assert dims == [[2, 60, 60], [4, 5, 15], [3, 20, 5], [5, 1, 1]]
    flat_src, flat_dst = x.reshape(-1), out.reshape(-1)
    sizes = [d[0] for d in dims]
    for e in range(p.numel()):
        rest, so, do = e, 0, 0
        for (n, a, b) in reversed(dims):
            c = rest % n
            rest //= n
            so += c * a
            do += c * b
        flat_dst[do] = flat_src[so]
    assert torch.equal(out, p.contiguous()) and sizes == [2, 4, 3, 5]
    row = x[1:2, :, 2:3].expand(2, 3, 4, 5)  # a broadcast along two axes
    dst = torch.empty(row.shape, dtype=x.dtype)
    assert _copy_dims(row.shape, row.stride(), dst.stride()) == [[2, 0, 60], [3, 20, 20],
                                                                  [4, 0, 5], [5, 1, 1]]
    assert _copy_dims((1, 1), (0, 0), (1, 1)) == [[1, 0, 0]]


@pytest.mark.parametrize("latent_shape", [(1, 8, 1, 1, 1), (2, 8, 3, 2, 4), (1, 8, 4, 5, 3)])
def test_working_shape_matches_the_oracle_decode(latent_shape):
    """x_t's working shape for latents that need no, some and all of the padding: the oracle
    decodes them and crops to (B, 3, 1 + (F - 1) * 8, H * 16, W * 16)."""
    cfg = mini_config()
    w = diffusion_decoder_weights(cfg, seed=5)
    latent = normal(latent_shape, seed=6, dtype=torch.float32)
    noise = normal(cfg.working_pixel_shape(latent_shape), seed=7)
    out = dref.decode(latent, noise, w, cfg)
    b, _, f, h, wd = latent_shape
    assert tuple(out.shape) == (b, 3, 1 + (f - 1) * 8, h * 16, wd * 16)


def test_copy_view_refusals():
    from kinomlx_b200 import ops

    a = torch.zeros((2, 3), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="shapes differ"):
        ops.copy_view(a, torch.zeros((3, 2), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bf16, fp16 or fp32"):
        ops.copy_view(a.to(torch.int32), torch.zeros((2, 3), dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA"):
        ops.copy_view(a, torch.zeros((2, 3), dtype=torch.float16))
