"""Host-side checks of the joint audio/video LTX-2 path (no GPU): the oracle's timestep wiring
against the reference's own A/V test, the device model's RoPE tables against the oracle's, and the
synthetic checkpoint's names."""

from __future__ import annotations

import torch

from oracle import ltx2 as ref
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.synthetic import ltx_av_weight_specs, make_weights

VIDEO = LTXVariant(dim=256, heads=2, context_dim=256, blocks=1)
AUDIO = LTXVariant(dim=128, heads=2, head_dim=64, context_dim=128, max_pos=(20,), blocks=1)


def _oracle_variant():
    pick = lambda v: ref.LTXVariant(dim=v.dim, heads=v.heads, head_dim=v.head_dim,
                                    context_dim=v.context_dim, max_pos=v.max_pos)
    return ref.LTXAVVariant(pick(VIDEO), pick(AUDIO))


def test_cross_scale_shift_follows_own_timesteps_and_gate_the_other_sigma():
    """tests/models/ltx2/transformer/test_model.py:242-266 of the reference, on the oracle: a
    stream's cross scale/shift changes with its own timestep only, its cross gate with the other
    modality's sigma only."""
    w = make_weights(ltx_av_weight_specs(VIDEO, AUDIO, 1), seed=3, dtype=torch.float32)
    v = _oracle_variant()
    base = ref.av_modulations(w, 0.5, 0.5, 1, v, torch.float32)
    own = ref.av_modulations(w, 0.25, 0.5, 1, v, torch.float32)  # video's own timestep moved
    other = ref.av_modulations(w, 0.5, 0.25, 1, v, torch.float32)  # audio's sigma moved
    assert not torch.equal(base["vcss"], own["vcss"])
    assert torch.equal(base["vcg"], own["vcg"])
    assert torch.equal(base["vcss"], other["vcss"])
    assert not torch.equal(base["vcg"], other["vcg"])
    assert not torch.equal(base["acg"], own["acg"]) and torch.equal(base["acss"], own["acss"])


def test_device_av_rope_tables_match_oracle():
    """The four RoPE table sets the device model prepares (video and audio self-attention, and
    the A/V attention's time-axis tables on the audio width with the larger max_pos) equal the
    oracle's bit for bit (kinomlx/models/ltx2/transformer/preprocessing.py:108-121, 190-200)."""
    w = make_weights(ltx_av_weight_specs(VIDEO, AUDIO, 1), seed=4)
    model = avm.LTXAVTransformer(w, VIDEO, AUDIO, "cpu")
    vpos = ref.pixel_coords(ref.patch_grid_bounds(2, 3, 4))
    start = torch.arange(9, dtype=torch.float32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    prep = model.prepare(torch.zeros(1, 3, VIDEO.dim), torch.zeros(1, 3, AUDIO.dim), vpos, apos)
    cross = (max(VIDEO.max_pos[0], AUDIO.max_pos[0]),)
    expect = {
        "video_pe": ref.precompute_freqs_cis(vpos, dim=VIDEO.dim, max_pos=VIDEO.max_pos, heads=VIDEO.heads),
        "audio_pe": ref.precompute_freqs_cis(apos, dim=AUDIO.dim, max_pos=AUDIO.max_pos, heads=AUDIO.heads),
        "video_cross_pe": ref.precompute_freqs_cis(vpos[:, 0:1], dim=AUDIO.dim, max_pos=cross, heads=VIDEO.heads),
        "audio_cross_pe": ref.precompute_freqs_cis(apos[:, 0:1], dim=AUDIO.dim, max_pos=cross, heads=AUDIO.heads),
    }
    for name, (cos, sin) in expect.items():
        got = getattr(prep, name)
        assert torch.equal(got.cos, cos) and torch.equal(got.sin, sin), name
    assert prep.audio_pe.cos.shape[-1] == 32  # 64-wide audio heads: half 32


def test_av_checkpoint_names_are_unique_and_complete():
    specs = ltx_av_weight_specs(VIDEO, AUDIO, 2)
    names = [s[0] for s in specs]
    assert len(names) == len(set(names))
    for needed in ("audio_patchify_proj.weight", "av_ca_v2a_gate_adaln_single.linear.weight",
                   "transformer_blocks.1.audio_to_video_attn.to_q.weight",
                   "transformer_blocks.1.scale_shift_table_a2v_ca_video", "audio_proj_out.bias"):
        assert needed in names
    shapes = dict((s[0], s[1]) for s in specs)
    assert shapes["transformer_blocks.0.audio_to_video_attn.to_q.weight"] == (AUDIO.dim, VIDEO.dim)
    assert shapes["transformer_blocks.0.video_to_audio_attn.to_k.weight"] == (AUDIO.dim, VIDEO.dim)
