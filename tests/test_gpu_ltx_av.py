"""The joint audio/video LTX-2 DiT on the device against the CPU oracle (kinomlx/models/ltx2/
transformer/transformer.py:225-413, model.py:577-635), bf16, same gates as the video-only tests:
relative L2 <= 1e-2, max relative error <= 2e-2 and cosine >= 0.999 for one forward, cosine >=
0.999 after a three-step trajectory.

Seeds: weights S, video latent S + 1, audio latent S + 2, video text S + 3, audio text S + 4.
Video positions are pixel-space patch bounds (scale 8/32/32, causal fix, 24 fps); audio
positions are 40 ms time bounds per token.
"""

from __future__ import annotations

import pytest
import torch

from oracle import fused_ops as rops
from oracle import ltx2 as ref
from kinomlx_b200 import ops
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.synthetic import ltx_av_weight_specs, make_weights, normal

pytestmark = pytest.mark.gpu


def _metrics(out, expect):
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return (float((o - e).norm() / e.norm()), float((o - e).abs().max() / e.abs().max()),
            float(torch.nn.functional.cosine_similarity(o, e, dim=0)))


def _oracle_variant(video: LTXVariant, audio: LTXVariant):
    pick = lambda v: ref.LTXVariant(dim=v.dim, heads=v.heads, head_dim=v.head_dim,
                                    context_dim=v.context_dim, max_pos=v.max_pos)
    return ref.LTXAVVariant(pick(video), pick(audio))


def _inputs(video, audio, seed, grid, ta, tc):
    f, h, w = grid
    weights = make_weights(ltx_av_weight_specs(video, audio, video.blocks), seed=seed)
    vlat = normal((1, f * h * w, video.in_channels), seed=seed + 1)
    alat = normal((1, ta, audio.in_channels), seed=seed + 2)
    vctx = normal((1, tc, video.dim), seed=seed + 3)
    actx = normal((1, tc - 2, audio.dim), seed=seed + 4)
    vpos = ref.pixel_coords(ref.patch_grid_bounds(f, h, w))
    start = torch.arange(ta, dtype=torch.float32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    return weights, vlat, alat, vctx, actx, vpos, apos


def test_split64_qk_norm_rope_matches_oracle(cuda_device):
    """Full-row RMSNorm over a 2048-wide row, then the split-half rotation of each 64-wide head
    (half 32) from (1, 32, T, 32) tables: the audio stream's and the A/V attention's q/k path."""
    audio = avm.audio_variant(1)
    start = torch.arange(37, dtype=torch.float32) * 0.04
    pos = torch.stack([start, start + 0.04], -1)[None, None]
    cos, sin = ref.precompute_freqs_cis(pos, dim=audio.dim, max_pos=audio.max_pos, heads=audio.heads)
    x = normal((2, 37, audio.dim), seed=40)
    wt = normal((audio.dim,), seed=41, std=0.1) + 1
    expect = ref.apply_split_rotary_emb(rops.rms_norm(x, wt, 1e-6), cos, sin)
    xd = x.to(cuda_device)
    ops.qk_norm_rope(xd, heads=audio.dim // 128, weight=wt.to(cuda_device),
                     norm=ops.QKNORM_FULL_ROW, rope=ops.ROPE_SPLIT64, cos=cos.to(cuda_device),
                     sin=sin.to(cuda_device), eps=1e-6)
    rel_l2, max_rel, cosine = _metrics(xd, expect)
    assert max_rel <= 2e-2 and cosine >= 0.9999, (rel_l2, max_rel, cosine)


def test_av_forward_full_width_matches_oracle(cuda_device):
    """One joint block at the reference's widths: video 4096 (32 x 128), audio 2048 (32 x 64);
    both streams' velocities against the oracle's."""
    video, audio = LTXVariant(blocks=1), avm.audio_variant(1)
    w, vlat, alat, vctx, actx, vpos, apos = _inputs(video, audio, 50, (2, 3, 8), 25, 12)
    sigma = ref.DISTILLED_STAGE_1_SIGMAS[5]
    ev, ea = ref.av_forward(w, vlat, alat, vctx, actx, sigma, vpos, apos,
                            _oracle_variant(video, audio), 1)
    model = avm.LTXAVTransformer(w, video, audio, cuda_device)
    prep = model.prepare(vctx, actx, vpos, apos)
    gv, ga = model.run(prep, vlat.to(cuda_device), alat.to(cuda_device), sigma)
    for out, exp in ((gv, ev), (ga, ea)):
        rel_l2, max_rel, cosine = _metrics(out, exp)
        assert rel_l2 <= 1e-2 and max_rel <= 2e-2 and cosine >= 0.999, (rel_l2, max_rel, cosine)


def test_av_denoise_matches_oracle(cuda_device):
    """Two joint blocks at video 1024 / audio 512 (8 heads each) over the last three distilled
    stage-1 steps, X0 + Euler fused into both final projections."""
    video = LTXVariant(dim=1024, heads=8, context_dim=1024, blocks=2)
    audio = LTXVariant(dim=512, heads=8, head_dim=64, context_dim=512, max_pos=(20,), blocks=2)
    w, vlat, alat, vctx, actx, vpos, apos = _inputs(video, audio, 60, (2, 4, 4), 20, 12)
    sigmas = ref.DISTILLED_STAGE_1_SIGMAS[5:]
    ev, ea = ref.av_denoise(w, vlat, alat, vctx, actx, vpos, apos, sigmas,
                            _oracle_variant(video, audio), 2)
    model = avm.LTXAVTransformer(w, video, audio, cuda_device)
    gv, ga = avm.denoise_av(model, vlat, alat, vctx, actx, vpos, apos, sigmas)
    for out, exp in ((gv, ev), (ga, ea)):
        rel_l2, max_rel, cosine = _metrics(out, exp)
        assert cosine >= 0.999 and rel_l2 <= 3e-2, (rel_l2, max_rel, cosine)
