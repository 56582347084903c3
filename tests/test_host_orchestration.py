"""Host-side orchestration of the model classes on the CPU: the kernel calls are replaced by torch
stand-ins of the same contracts (tests/stand_in_kernels.py), so these tests check only what the
classes hand to which kernel (slices, aliasing, modulation rows, RoPE tables, step order) against
the oracle. Covered: the fp32 Flux2 and LTX-2 transformers, the fp32 VAE decoder and the joint
audio/video LTX-2 model (run in fp32 here). The bf16 Flux2 class fuses the QK norm and the lead
rows into its GEMM epilogues, which the stand-ins do not model; it and every kernel are tested on
the GPU."""

from __future__ import annotations

import torch

import stand_in_kernels as stand_in
from oracle import flux2 as fref
from oracle import ltx2 as lref
from oracle import video_vae as vref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import rotary_positions
from kinomlx_b200.flux2.transformer_f32 import Flux2TransformerF32
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2 import video_vae as vae
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.ltx2.transformer_f32 import LTXVideoTransformerF32
from kinomlx_b200.ltx2.video_vae_f32 import VideoDecoderF32
from kinomlx_b200.synthetic import (flux_weights, ltx_av_weight_specs, ltx_weights, make_weights,
                                    normal)

F32 = torch.float32
CPU = torch.device("cpu")
TOL = 1e-5  # the stand-ins compute what the oracle computes: only the wiring can differ


def _max_rel(out, expect) -> float:
    return float((out.float() - expect.float()).abs().max() / expect.float().abs().max())


def _flux_variant(mlp: str) -> fcfg.FluxVariant:
    return fcfg.FluxVariant(dim=256, heads=2, mlp=mlp, mlp_hidden=512, rope_axes=(64, 64),
                            rope_theta=10000.0, in_channels=32, context_dim=64, double_blocks=1,
                            single_blocks=1)


def test_flux_f32_blocks_and_cfg_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    for mlp in ("gelu_tanh", "swiglu"):
        v = _flux_variant(mlp)
        w = flux_weights(v, seed=70, dtype=F32)
        nt, h, wd = 16, 4, 6
        ids = torch.cat([torch.zeros((1, nt, 2), dtype=torch.int64), fref.image_ids(h, wd, 2)], 1)
        image, text = normal((2, h * wd, v.dim), seed=71, dtype=F32), normal((2, nt, v.dim), seed=72, dtype=F32)
        t = torch.tensor([0.25, 0.75])
        cos4, sin4 = fref.rotary_positions(ids, v)
        emb = fref.timestep_embedding(w, t * 1000)
        im = fref.modulation(w, "double_stream_modulation_img", emb)
        tm = fref.modulation(w, "double_stream_modulation_txt", emb)
        exp_img, exp_txt = fref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)
        model = Flux2TransformerF32(w, v, CPU)
        cos, sin = rotary_positions(ids, v)
        img, txt = model.double_block(0, image, text, t * 1000, cos, sin)
        assert _max_rel(img, exp_img) < TOL and _max_rel(txt, exp_txt) < TOL
        sm = fref.modulation(w, "single_stream_modulation", emb)
        value = torch.cat([text, image], 1)
        expect = fref.single_block(w, 0, value, sm, cos4, sin4, v)
        assert _max_rel(model.single_block(0, value, nt, t * 1000, cos, sin), expect) < TOL
        noise = normal((1, h * wd, v.in_channels), seed=73, dtype=F32)
        ctx, neg = normal((1, nt, v.context_dim), seed=74, dtype=F32), normal((1, nt, v.context_dim), seed=75, dtype=F32)
        sig = fref.linear_sigmas(2)
        expect = fref.denoise(w, noise, ctx, ids, sig, v, negative=neg, guidance=3.0)
        out = sampling.denoise(model, noise, ctx, ids, sigmas=sampling.linear_sigmas(2),
                               negative=neg, guidance=3.0)
        assert _max_rel(out, expect) < TOL


def test_ltx_f32_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    v = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    w = ltx_weights(v, seed=76, dtype=F32)
    latent = normal((2, 2 * 3 * 4, v.in_channels), seed=77, dtype=F32)
    context = normal((2, 6, v.context_dim), seed=78, dtype=F32)
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = lref.denoise(w, latent, context, pos, sigmas, v)
    out = ldn.denoise_loop(LTXVideoTransformerF32(w, v, CPU), latent, context, pos, sigmas)
    assert _max_rel(out, expect) < TOL


def test_vae_f32_tiled_decode(monkeypatch):
    stand_in.install(monkeypatch)
    blocks = (("res", 1), ("d2s", (2, 2, 2), 2), ("res", 1), ("d2s", (1, 2, 2), 1), ("res", 1))
    for norm, causal in (("pixel", False), ("group32", True)):
        v = vae.VaeVariant(norm=norm, causal=causal, top_width=64, blocks=blocks)
        rv = vref.VaeVariant(norm=norm, causal=causal, top_width=64, blocks=blocks)
        w = make_weights(vae.vae_weight_specs(v), seed=79, dtype=F32)
        latent = normal((1, 128, 2, 5, 7), seed=80, dtype=F32)
        expect = vref.decode_tiled(w, latent, rv, tile=3, overlap=1, scale=16, dtype=F32)
        out = VideoDecoderF32(w, v, CPU).decode(latent, tile=3, overlap=1)
        assert _max_rel(out, expect) < TOL


def test_av_model_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    monkeypatch.setattr(avm, "BF", F32)  # run the bf16 model's wiring in fp32
    video = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    audio = LTXVariant(dim=128, heads=2, head_dim=64, context_dim=128, max_pos=(20,), blocks=2)
    w = make_weights(ltx_av_weight_specs(video, audio, 2), seed=81, dtype=F32)
    vlat = normal((1, 2 * 3 * 4, video.in_channels), seed=82, dtype=F32)
    alat = normal((1, 10, audio.in_channels), seed=83, dtype=F32)
    vctx, actx = normal((1, 6, video.dim), seed=84, dtype=F32), normal((1, 5, audio.dim), seed=85, dtype=F32)
    vpos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    start = torch.arange(10, dtype=F32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    pick = lambda x: lref.LTXVariant(dim=x.dim, heads=x.heads, head_dim=x.head_dim,
                                     context_dim=x.context_dim, max_pos=x.max_pos)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    ev, ea = lref.av_denoise(w, vlat, alat, vctx, actx, vpos, apos, sigmas,
                             lref.LTXAVVariant(pick(video), pick(audio)), 2)
    gv, ga = avm.denoise_loop(avm.LTXAVTransformer(w, video, audio, CPU), vlat, alat, vctx,
                              actx, vpos, apos, sigmas)
    assert _max_rel(gv, ev) < TOL and _max_rel(ga, ea) < TOL
