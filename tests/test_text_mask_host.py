"""Padded text masks of the LTX-2 cross-attention on the CPU (no GPU).

The reference turns a text context mask into an additive bias on the cross-attention's scores
(kinomlx/models/ltx2/transformer/preprocessing.py:85-96; attention.py:164-186): a floating-point
mask is the bias itself in the compute dtype, any other mask becomes (mask - 1) * -min(dtype).
The reference's tests hold no known answer for a padded prompt, so the oracle is pinned by the
properties that rule makes exact: an all-ones mask changes nothing, and masking the trailing
tokens equals cutting them from the context. The device classes' mask handling (the key-bias
operand, its plumbing into the video, fp32 and joint audio/video classes and the reference's
`denoise_loop`) is then checked against the oracle with the kernels replaced by the torch
stand-ins of tests/stand_in_kernels.py; the kernels themselves are tested on the GPU."""

from __future__ import annotations

import pytest
import torch

import stand_in_kernels as stand_in
from oracle import ltx2 as lref
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer, context_key_bias
from kinomlx_b200.ltx2.transformer_f32 import LTXVideoTransformerF32
from kinomlx_b200.synthetic import ltx_av_weight_specs, ltx_weights, make_weights, normal
from test_host_orchestration import _kaiming, _max_rel

F32 = torch.float32
CPU = torch.device("cpu")
TOL = 1e-5
MIN = -3.3895313892515355e38


def _padding_mask(batch: int, tokens: int, valid: list[int], dtype=torch.int32) -> torch.Tensor:
    m = torch.zeros((batch, tokens), dtype=dtype)
    for b, n in enumerate(valid):
        m[b, :n] = 1
    return m


# ----------------------------------------------------------------------------- oracle pins
def test_oracle_mask_bias_values():
    m = _padding_mask(2, 5, [5, 3])
    bias = lref.context_mask_bias(m, torch.bfloat16)
    assert bias.shape == (2, 1, 1, 5) and bias.dtype == torch.bfloat16
    assert torch.equal(bias[0].float(), torch.zeros(1, 1, 5))
    assert torch.equal(bias[1, 0, 0].float(), torch.tensor([0.0, 0.0, 0.0, MIN, MIN]))
    assert float(lref.context_mask_bias(m, torch.float16)[1, 0, 0, 4]) == -65504.0
    f = torch.tensor([[0.0, -2.5, -1e4]])
    assert torch.equal(lref.context_mask_bias(f, torch.float32)[0, 0, 0], f[0])
    assert lref.context_mask_bias(f[:, None].expand(1, 4, 3), F32).shape == (1, 1, 4, 3)


def _oracle_case(seed: int):
    v = lref.LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    w = _kaiming(ltx_weights(LTXVariant(dim=256, heads=2, context_dim=256, blocks=2), seed=seed,
                             dtype=F32))
    latent = normal((2, 2 * 3 * 4, v.in_channels), seed=seed + 1, dtype=F32)
    context = normal((2, 7, v.context_dim), seed=seed + 2, dtype=F32)
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    return v, w, latent, context, pos


def test_oracle_all_ones_mask_is_no_mask_and_padding_is_truncation():
    v, w, latent, context, pos = _oracle_case(200)
    plain = lref.forward(w, latent, context, 0.725, pos, v, dtype=F32)
    ones = lref.forward(w, latent, context, 0.725, pos, v, dtype=F32,
                        context_mask=torch.ones((2, 7), dtype=torch.int64))
    assert torch.equal(plain, ones)
    masked = lref.forward(w, latent, context, 0.725, pos, v, dtype=F32,
                          context_mask=_padding_mask(2, 7, [4, 4]))
    cut = lref.forward(w, latent, context[:, :4], 0.725, pos, v, dtype=F32)
    assert _max_rel(masked, cut) < 1e-6
    assert _max_rel(masked, plain) > 1e-3  # the padding tokens did take part without the mask


# ----------------------------------------------------------------------------- host operand
def test_context_key_bias_matches_the_oracle_bias():
    for mask in (_padding_mask(2, 6, [6, 2]), _padding_mask(2, 6, [1, 5], torch.bool),
                 torch.tensor([[0.0, -1.5, -3.0, 0.25, -7.0, 0.0]]).expand(2, 6)):
        for dtype in (torch.bfloat16, F32):
            got = context_key_bias(mask, 2, 6, CPU, dtype)
            expect = lref.context_mask_bias(mask, dtype).float().reshape(2, 6)
            assert got.shape == (2, 8) and got.dtype == F32
            assert torch.equal(got[:, :6], expect) and torch.equal(got[:, 6:], torch.zeros(2, 2))
    one = context_key_bias(_padding_mask(1, 5, [3]), 3, 5, CPU)  # one mask for every prompt
    assert torch.equal(one[0], one[2]) and float(one[1, 4]) == MIN
    assert context_key_bias(None, 2, 6, CPU) is None


def test_context_key_bias_refusals():
    with pytest.raises(ValueError, match="per-query masks"):
        context_key_bias(torch.ones(1, 4, 6), 1, 6, CPU)
    with pytest.raises(ValueError, match="does not match"):
        context_key_bias(torch.ones(1, 5), 1, 6, CPU)
    with pytest.raises(ValueError, match="hold 1"):
        context_key_bias(torch.full((1, 6), 2), 1, 6, CPU)


# ----------------------------------------------------------------------------- classes
def test_video_classes_with_padded_masks_match_oracle(monkeypatch):
    stand_in.install(monkeypatch)
    v, w, latent, context, pos = _oracle_case(210)
    dv = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    mask = _padding_mask(2, 7, [3, 6])
    expect = lref.denoise(w, latent, context, pos, sigmas, v, context_mask=mask)
    for cls in (LTXVideoTransformer, LTXVideoTransformerF32):
        model = cls(w, dv, CPU)
        out = ldn.denoise_video(model, latent, context, pos, sigmas, context_mask=mask)
        assert _max_rel(out - latent, expect - latent) < TOL, cls.__name__
    # the reference surface: denoise_loop(..., video_context_mask=)
    state = ldn.LatentState(latent=latent.clone(), denoise_mask=None, positions=pos)
    video, _ = ldn.denoise_loop(state, None, sigmas, transformer=LTXVideoTransformer(w, dv, CPU),
                                video_context=context, video_context_mask=mask)
    assert _max_rel(video.latent - latent, expect - latent) < TOL
    unmasked = lref.denoise(w, latent, context, pos, sigmas, v)
    assert _max_rel(unmasked - latent, expect - latent) > 1e-3


def test_av_class_with_padded_masks_matches_oracle(monkeypatch):
    stand_in.install(monkeypatch)
    monkeypatch.setattr(avm, "BF", F32)
    video = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    audio = LTXVariant(dim=128, heads=2, head_dim=64, context_dim=128, max_pos=(20,), blocks=2)
    w = _kaiming(make_weights(ltx_av_weight_specs(video, audio, 2), seed=220, dtype=F32))
    vlat = normal((1, 2 * 3 * 4, video.in_channels), seed=221, dtype=F32)
    alat = normal((1, 10, audio.in_channels), seed=222, dtype=F32)
    vctx, actx = normal((1, 6, video.dim), seed=223, dtype=F32), normal((1, 5, audio.dim), seed=224, dtype=F32)
    vpos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    start = torch.arange(10, dtype=F32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    pick = lambda x: lref.LTXVariant(dim=x.dim, heads=x.heads, head_dim=x.head_dim,
                                     context_dim=x.context_dim, max_pos=x.max_pos)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    vmask, amask = _padding_mask(1, 6, [4]), _padding_mask(1, 5, [2], torch.bool)
    ev, ea = lref.av_denoise(w, vlat, alat, vctx, actx, vpos, apos, sigmas,
                             lref.LTXAVVariant(pick(video), pick(audio)), 2,
                             video_context_mask=vmask, audio_context_mask=amask)
    gv, ga = avm.denoise_av(avm.LTXAVTransformer(w, video, audio, CPU), vlat, alat, vctx, actx,
                            vpos, apos, sigmas, video_context_mask=vmask, audio_context_mask=amask)
    assert _max_rel(gv - vlat, ev - vlat) < TOL and _max_rel(ga - alat, ea - alat) < TOL
