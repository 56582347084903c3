"""Host-side orchestration of the model classes on the CPU: the kernel calls are replaced by torch
stand-ins of the same contracts (tests/stand_in_kernels.py), so these tests check only what the
classes hand to which kernel (slices, aliasing, modulation rows, RoPE tables, step order) against
the oracle. Covered: the fp32 Flux2 and LTX-2 transformers, the fp32 VAE decoder, and the bf16
Flux2, LTX-2 video and joint audio/video classes (run in fp32 here; the stand-in GEMM applies the
fused QK-norm/RoPE, lead-row and SwiGLU epilogues the way the kernel does), with the Flux2 CFG,
in-context reference and KV-editing loops. Weights are rescaled so that a wiring mistake moves
the compared update by far more than the tolerance (see `_kaiming`). Every kernel is tested on
the GPU."""

from __future__ import annotations

import torch

import stand_in_kernels as stand_in
from oracle import flux2 as fref
from oracle import ltx2 as lref
from oracle import video_vae as vref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import Flux2Transformer, rotary_positions
from kinomlx_b200.flux2.transformer_f32 import Flux2TransformerF32
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2 import video_vae as vae
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.ltx2.transformer_f32 import LTXVideoTransformerF32
from kinomlx_b200.ltx2.video_vae_f32 import VideoDecoderF32
from kinomlx_b200.synthetic import (flux_weights, ltx_av_weight_specs, ltx_weights, make_weights,
                                    normal)

F32 = torch.float32
CPU = torch.device("cpu")
TOL = 1e-5  # the stand-ins compute what the oracle computes: only the wiring can differ


def _max_rel(out, expect) -> float:
    return float((out.float() - expect.float()).abs().max() / expect.float().abs().max())


def _kaiming(w: dict) -> dict:
    """Projection weights rescaled to std 1/sqrt(fan_in) (modulations x4) and norm weights moved
    off 1: the synthetic std 0.02 leaves gates near 0.02, where a wiring mistake moves the output
    by less than the tolerance, and all-ones norm weights hide a swapped norm."""
    scaled = {}
    for name, t in w.items():
        if t.dim() == 2 and name.endswith(".weight") and "norm" not in name:
            t = t / t.std() * t.shape[1] ** -0.5 * (4.0 if "modulation" in name else 1.0)
        elif t.dim() == 1 and "norm" in name:
            t = t + 0.2 * normal(t.shape, seed=len(scaled), dtype=t.dtype)
        scaled[name] = t
    return scaled


def _flux_variant(mlp: str) -> fcfg.FluxVariant:
    return fcfg.FluxVariant(dim=256, heads=2, mlp=mlp, mlp_hidden=512, rope_axes=(64, 64),
                            rope_theta=10000.0, in_channels=32, context_dim=64, double_blocks=1,
                            single_blocks=1)


def test_flux_f32_blocks_and_cfg_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    for mlp in ("gelu_tanh", "swiglu"):
        v = _flux_variant(mlp)
        w = _kaiming(flux_weights(v, seed=70, dtype=F32))
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
        out = sampling.denoise_joint(model, noise, ctx, ids, sigmas=sampling.linear_sigmas(2),
                               negative=neg, guidance=3.0)
        assert _max_rel(out - noise, expect - noise) < TOL


def test_flux_f32_in_context_references(monkeypatch):
    """The fp32 class under the in-context reference loop: [target | reference] rows, the target
    rows' velocity only, with and without CFG."""
    stand_in.install(monkeypatch)
    v, w, text_ids = _flux_case("gelu_tanh", 16, 130)
    noise = normal((1, 12, v.in_channels), seed=131, dtype=F32)
    refs = normal((1, 6, v.in_channels), seed=132, dtype=F32)
    ctx, neg = normal((1, 16, v.context_dim), seed=133, dtype=F32), normal((1, 16, v.context_dim), seed=134, dtype=F32)
    ref_ids = fref.image_ids(2, 3, 4)
    ref_ids[..., 0] = 10
    ids = torch.cat([text_ids, fref.image_ids(3, 4, 4), ref_ids], 1)
    model = Flux2TransformerF32(w, v, CPU)
    for negative, g in ((None, 1.0), (neg, 2.5)):
        expect = fref.denoise(w, noise, ctx, ids, fref.linear_sigmas(2), v, negative=negative,
                              guidance=g, references=refs)
        out = sampling.denoise_joint(model, noise, ctx, ids, sigmas=sampling.linear_sigmas(2),
                               negative=negative, guidance=g, references=refs)
        assert _max_rel(out - noise, expect - noise) < TOL


def test_ltx_f32_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    v = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    w = _kaiming(ltx_weights(v, seed=76, dtype=F32))
    latent = normal((2, 2 * 3 * 4, v.in_channels), seed=77, dtype=F32)
    context = normal((2, 6, v.context_dim), seed=78, dtype=F32)
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = lref.denoise(w, latent, context, pos, sigmas, v)
    out = ldn.denoise_video(LTXVideoTransformerF32(w, v, CPU), latent, context, pos, sigmas)
    assert _max_rel(out - latent, expect - latent) < TOL


def test_ltx_bf16_class_trajectory(monkeypatch):
    """The bf16 LTX-2 video class's wiring (run in fp32): AdaLN tables, gated self- and
    cross-attention with full-row QK norms and split RoPE, prompt AdaLN, X0 + Euler output."""
    stand_in.install(monkeypatch)
    v = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    w = _kaiming(ltx_weights(v, seed=120, dtype=F32))
    latent = normal((2, 2 * 3 * 4, v.in_channels), seed=121, dtype=F32)
    context = normal((2, 6, v.context_dim), seed=122, dtype=F32)
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = lref.denoise(w, latent, context, pos, sigmas, v)
    out = ldn.denoise_video(LTXVideoTransformer(w, v, CPU), latent, context, pos, sigmas)
    assert _max_rel(out - latent, expect - latent) < TOL


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


def test_vae_bf16_class_tiled_decode(monkeypatch):
    """The bf16 decoder's wiring (run in fp32): each GroupNorm normalises with the statistics the
    conv that produced its input kept in its epilogue (the stand-in norm reads only those), the
    residual conv writes over its residual, depth-to-space rows, the tiled blend."""
    stand_in.install(monkeypatch)
    blocks = (("res", 1), ("d2s", (2, 2, 2), 2), ("res", 2), ("d2s", (1, 2, 2), 1), ("res", 1))
    for norm, causal in (("pixel", True), ("group32", False)):
        v = vae.VaeVariant(norm=norm, causal=causal, top_width=64, blocks=blocks)
        rv = vref.VaeVariant(norm=norm, causal=causal, top_width=64, blocks=blocks)
        w = make_weights(vae.vae_weight_specs(v), seed=123, dtype=F32)
        w = {k: (t + 0.1 * normal(t.shape, seed=124, dtype=F32) if "norm" in k else t) for k, t in w.items()}
        latent = normal((1, 128, 2, 5, 7), seed=125, dtype=F32)
        expect = vref.decode_tiled(w, latent, rv, tile=3, overlap=1, scale=16, dtype=F32)
        out = vae.VideoDecoder(w, v, CPU).decode(latent, tile=3, overlap=1)
        assert _max_rel(out, expect) < TOL


def test_av_model_trajectory(monkeypatch):
    stand_in.install(monkeypatch)
    monkeypatch.setattr(avm, "BF", F32)  # run the bf16 model's wiring in fp32
    video = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    audio = LTXVariant(dim=128, heads=2, head_dim=64, context_dim=128, max_pos=(20,), blocks=2)
    w = _kaiming(make_weights(ltx_av_weight_specs(video, audio, 2), seed=81, dtype=F32))
    vlat = normal((1, 2 * 3 * 4, video.in_channels), seed=82, dtype=F32)
    alat = normal((1, 10, audio.in_channels), seed=83, dtype=F32)
    vctx, actx = normal((1, 6, video.dim), seed=84, dtype=F32), normal((1, 5, audio.dim), seed=85, dtype=F32)
    vpos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    start = torch.arange(10, dtype=F32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    pick = lambda x: lref.LTXVariant(dim=x.dim, heads=x.heads, head_dim=x.head_dim,
                                     context_dim=x.context_dim, max_pos=x.max_pos)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    # a gate scale apart from the timestep scale (both 1000 by default) tells the two apart
    ev, ea = lref.av_denoise(w, vlat, alat, vctx, actx, vpos, apos, sigmas,
                             lref.LTXAVVariant(pick(video), pick(audio), av_gate_scale=250.0), 2)
    gv, ga = avm.denoise_av(avm.LTXAVTransformer(w, video, audio, CPU, av_gate_scale=250.0),
                              vlat, alat, vctx, actx, vpos, apos, sigmas)
    assert _max_rel(gv - vlat, ev - vlat) < TOL and _max_rel(ga - alat, ea - alat) < TOL


def _flux_case(mlp: str, nt: int, seed: int, single_blocks: int = 1):
    v = fcfg.FluxVariant(dim=256, heads=2, mlp=mlp, mlp_hidden=512, rope_axes=(32, 32, 32, 32),
                         rope_theta=2000.0, in_channels=32, context_dim=64, double_blocks=1,
                         single_blocks=single_blocks)
    w = _kaiming(flux_weights(v, seed=seed, dtype=F32))
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    return v, w, text_ids


def test_flux_bf16_class_blocks_cfg_and_references(monkeypatch):
    """The bf16 class's wiring: the split double block (16 text rows) and the joint one (256 text
    rows, text weights as lead rows), the single block, the CFG loop and in-context references
    appended after the target rows."""
    stand_in.install(monkeypatch)
    for mlp, nt in (("gelu_tanh", 16), ("swiglu", 16), ("swiglu", 256)):
        v, w, text_ids = _flux_case(mlp, nt, 100)
        h, wd = 3, 4
        ids = torch.cat([text_ids, fref.image_ids(h, wd, 4)], 1)
        image, text = normal((2, h * wd, v.dim), seed=101, dtype=F32), normal((2, nt, v.dim), seed=102, dtype=F32)
        t = torch.tensor([0.25, 0.75])
        cos4, sin4 = fref.rotary_positions(ids, v)
        emb = fref.timestep_embedding(w, t * 1000)
        im = fref.modulation(w, "double_stream_modulation_img", emb)
        tm = fref.modulation(w, "double_stream_modulation_txt", emb)
        exp_img, exp_txt = fref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)
        model = Flux2Transformer(w, v, CPU)
        cos, sin = rotary_positions(ids, v)
        img, txt = model.double_block(0, image, text, t * 1000, cos, sin)
        assert _max_rel(img, exp_img) < TOL and _max_rel(txt, exp_txt) < TOL
        sm = fref.modulation(w, "single_stream_modulation", emb)
        value = torch.cat([text, image], 1)
        expect = fref.single_block(w, 0, value, sm, cos4, sin4, v)
        assert _max_rel(model.single_block(0, value, nt, t * 1000, cos, sin), expect) < TOL
        noise = normal((1, h * wd, v.in_channels), seed=103, dtype=F32)
        ctx, neg = normal((1, nt, v.context_dim), seed=104, dtype=F32), normal((1, nt, v.context_dim), seed=105, dtype=F32)
        sig = fref.linear_sigmas(2)
        expect = fref.denoise(w, noise, ctx, ids, sig, v, negative=neg, guidance=3.0)
        out = sampling.denoise_joint(model, noise, ctx, ids, sigmas=sampling.linear_sigmas(2),
                               negative=neg, guidance=3.0)
        assert _max_rel(out - noise, expect - noise) < TOL
        refs = normal((1, 6, v.in_channels), seed=106, dtype=F32)
        ref_ids = fref.image_ids(2, 3, 4)
        ref_ids[..., 0] = 10
        ids_r = torch.cat([ids, ref_ids], 1)
        for negative, g in ((None, 1.0), (neg, 2.0)):
            expect = fref.denoise(w, noise, ctx, ids_r, sig, v, negative=negative, guidance=g,
                                  references=refs)
            out = sampling.denoise_joint(model, noise, ctx, ids_r, sigmas=sampling.linear_sigmas(2),
                                   negative=negative, guidance=g, references=refs)
            assert out.shape == noise.shape and _max_rel(out - noise, expect - noise) < TOL


def test_flux_bf16_class_kv_editing_trajectory(monkeypatch):
    """KV editing on the bf16 class's wiring: extraction over [text | reference | target] rows
    (reference rows on the timestep-0 modulations, their queries on reference keys only), reuse
    with the kept rows as a second key segment, with and without per-step recomputation, on the
    split (16 text rows) and joint (256) double-block paths; the cache is closed afterwards."""
    stand_in.install(monkeypatch)
    kept = []
    for mlp, nt in (("swiglu", 16), ("gelu_tanh", 256)):
        v, w, text_ids = _flux_case(mlp, nt, 110, single_blocks=2)
        h, wd = 3, 4
        image_ids = fref.image_ids(h, wd, 4)
        ref_ids = fref.image_ids(2, 3, 4)
        ref_ids[..., 0] = 10
        noise = normal((1, h * wd, v.in_channels), seed=111, dtype=F32)
        refs = normal((1, 6, v.in_channels), seed=112, dtype=F32)
        ctx = normal((1, nt, v.context_dim), seed=113, dtype=F32)
        sig = fref.linear_sigmas(3)
        model = Flux2Transformer(w, v, CPU)
        made = model.new_reference_kv
        monkeypatch.setattr(model, "new_reference_kv", lambda n: kept.append(made(n)) or kept[-1])
        for recompute in (False, True):
            expect = fref.denoise_kv(w, noise, ctx, text_ids, image_ids, refs, ref_ids, sig, v,
                                     recompute=recompute)
            out = sampling.denoise_kv(model, noise, ctx, text_ids, image_ids, refs, ref_ids,
                                      sigmas=sampling.linear_sigmas(3),
                                      recompute_reference_kv=recompute)
            assert out.shape == noise.shape and _max_rel(out - noise, expect - noise) < TOL
    assert len(kept) == 2 * (1 + 3) and all(c.closed for c in kept)
