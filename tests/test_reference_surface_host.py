"""The reference-signature call sites on the CPU, kernels replaced by the torch stand-ins of
tests/stand_in_kernels.py: the Klein `denoise(model, noise, text, image_ids, text_ids, *,
recipe, references, reference_ids, negative, reporter, on_step)` of
kinomlx/models/flux2/sampling.py:116-281 and its `SamplingRecipe`; the LTX-2 `denoise_step` /
`denoise_loop(video_state, audio_state, sigmas, *, transformer, video_context, ...)` of
kinomlx/models/ltx2/denoise.py:159-365; the argument contracts of `WinogradConv3d` and the
Euler steps. Each loop is checked against the oracle, and each refusal against the reference's
message."""

from __future__ import annotations

import pytest
import torch

import stand_in_kernels as stand_in
from oracle import flux2 as fref
from oracle import ltx2 as lref
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.sampling import Flux2CFGMode, Flux2Variant, SamplingRecipe
from kinomlx_b200.flux2.transformer import Flux2Transformer
from kinomlx_b200.kernels.winograd_conv3d import WinogradConv3d
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.samplers import steps
from kinomlx_b200.synthetic import ltx_weights, normal
from test_host_orchestration import _flux_case, _kaiming, _max_rel

F32 = torch.float32
CPU = torch.device("cpu")
TOL = 1e-5


# ----------------------------------------------------------------------------- recipe
def test_recipe_profiles_and_rules():
    assert SamplingRecipe().resolved() == (4, 1.0)
    assert SamplingRecipe(variant=Flux2Variant.BASE).resolved() == (50, 4.0)
    assert SamplingRecipe(variant="kv").resolved() == (4, 1.0)
    assert SamplingRecipe(sigmas=(1.0, 0.5, 0.0), steps=9).resolved()[0] == 2
    assert SamplingRecipe(variant="base", steps=3, guidance=2.5,
                          cfg_mode=Flux2CFGMode.BATCHED).resolved() == (3, 2.5)
    with pytest.raises(ValueError, match="requires the KV recipe"):
        SamplingRecipe(recompute_reference_kv=True).resolved()
    with pytest.raises(ValueError, match="base recipe only"):
        SamplingRecipe(guidance=2.0).resolved()
    with pytest.raises(ValueError, match="requires the base model"):
        SamplingRecipe(cfg_mode="batched").resolved()
    with pytest.raises(ValueError, match="decrease strictly"):
        SamplingRecipe(sigmas=(1.0, 1.0, 0.0)).resolved()
    with pytest.raises(ValueError, match="between 0 and 1"):
        SamplingRecipe(sigmas=(1.5, 0.0)).resolved()
    # explicit sigmas are kept (fp32); otherwise the Klein shift of the target grid
    assert torch.equal(SamplingRecipe(sigmas=(1.0, 0.25, 0.0)).sigma_array(64),
                       torch.tensor([1.0, 0.25, 0.0]))
    assert torch.equal(SamplingRecipe().sigma_array(4096), fref.schedule(4096, 4))


# ----------------------------------------------------------------------------- Klein denoise
def _klein(monkeypatch):
    stand_in.install(monkeypatch)
    v, w, text_ids = _flux_case("gelu_tanh", 16, 140)
    image_ids = fref.image_ids(3, 4, 4)
    noise = normal((1, 12, v.in_channels), seed=141, dtype=F32)
    ctx = normal((1, 16, v.context_dim), seed=142, dtype=F32)
    neg = normal((1, 16, v.context_dim), seed=143, dtype=F32)
    return v, w, text_ids, image_ids, noise, ctx, neg


def test_klein_denoise_reference_signature_matches_oracle(monkeypatch):
    v, w, text_ids, image_ids, noise, ctx, neg = _klein(monkeypatch)
    model = Flux2Transformer(w, v, CPU)
    ids = torch.cat([text_ids, image_ids], 1)
    sig = (1.0, 0.5, 0.0)
    expect = fref.denoise(w, noise, ctx, ids, torch.tensor(sig), v)
    out = sampling.denoise(model, noise, ctx, image_ids, text_ids, recipe=SamplingRecipe(sigmas=sig))
    assert _max_rel(out - noise, expect - noise) < TOL
    # guidance 2.5 on the base recipe, both CFG modes, equal to the oracle's batched CFG
    expect = fref.denoise(w, noise, ctx, ids, torch.tensor(sig), v, negative=neg, guidance=2.5)
    for mode in (Flux2CFGMode.SEQUENTIAL, Flux2CFGMode.BATCHED):
        recipe = SamplingRecipe(variant="base", guidance=2.5, cfg_mode=mode, sigmas=sig)
        out = sampling.denoise(model, noise, ctx, image_ids, text_ids, recipe=recipe, negative=neg)
        assert _max_rel(out - noise, expect - noise) < TOL, mode
    # in-context references ([target | reference] rows; target rows updated)
    refs = normal((1, 6, v.in_channels), seed=144, dtype=F32)
    ref_ids = fref.image_ids(2, 3, 4)
    ref_ids[..., 0] = 10
    expect = fref.denoise(w, noise, ctx, torch.cat([ids, ref_ids], 1), torch.tensor(sig), v,
                          references=refs)
    out = sampling.denoise(model, noise, ctx, image_ids, text_ids, recipe=SamplingRecipe(sigmas=sig),
                           references=refs, reference_ids=ref_ids)
    assert out.shape == noise.shape and _max_rel(out - noise, expect - noise) < TOL
    # the KV recipe with references: extraction then reuse, as the oracle's KV loop
    expect = fref.denoise_kv(w, noise, ctx, text_ids, image_ids, refs, ref_ids,
                             torch.tensor(sig), v)
    out = sampling.denoise(model, noise, ctx, image_ids, text_ids,
                           recipe=SamplingRecipe(variant="kv", sigmas=sig),
                           references=refs, reference_ids=ref_ids)
    assert _max_rel(out - noise, expect - noise) < TOL


def test_klein_denoise_on_step_reporter_and_inputs_untouched(monkeypatch):
    v, w, text_ids, image_ids, noise, ctx, _ = _klein(monkeypatch)
    model = Flux2Transformer(w, v, CPU)
    sig = (1.0, 0.75, 0.25, 0.0)
    plain = sampling.denoise(model, noise, ctx, image_ids, text_ids, recipe=SamplingRecipe(sigmas=sig))
    seen, phases = [], []

    class Reporter:
        def phase_start(self, name, total, unit):
            phases.append(("start", name, total, unit))

        def phase_advance(self, name):
            phases.append(("advance", name))

        def phase_end(self, name):
            phases.append(("end", name))

    before = noise.clone()
    out = sampling.denoise(model, noise, ctx, image_ids, text_ids, recipe=SamplingRecipe(sigmas=sig),
                           reporter=Reporter(),
                           on_step=lambda i, cur, vel: seen.append((i, cur.clone(), vel.clone())))
    assert torch.equal(noise, before)
    assert [i for i, _, _ in seen] == [0, 1, 2]
    assert torch.equal(seen[-1][1], out) and _max_rel(out, plain) < TOL
    # each step's latent is the previous one plus dt times the velocity handed to on_step
    prev = noise
    for i, cur, vel in seen:
        expect = fref.euler_step(prev, vel, torch.tensor(sig[i + 1] - sig[i]))
        assert _max_rel(cur - prev, expect - prev) < TOL
        prev = cur
    assert phases[0] == ("start", "denoise", 3, "step") and phases[-1] == ("end", "denoise")
    assert phases.count(("advance", "denoise")) == 3


def test_klein_denoise_names_the_nonfinite_step(monkeypatch):
    v, w, text_ids, image_ids, noise, ctx, _ = _klein(monkeypatch)
    model = Flux2Transformer(w, v, CPU)
    run, calls = model.run, []

    def poisoned(*args, **kwargs):
        out = run(*args, **kwargs)
        calls.append(1)
        if len(calls) == 2:
            out.fill_(float("nan"))
        return out

    monkeypatch.setattr(model, "run", poisoned)
    with pytest.raises(FloatingPointError, match="nonfinite latents at step 2"):
        sampling.denoise(model, noise, ctx, image_ids, text_ids,
                         recipe=SamplingRecipe(sigmas=(1.0, 0.75, 0.25, 0.0)))
    assert len(calls) == 2


def test_klein_denoise_refusals(monkeypatch):
    v, w, text_ids, image_ids, noise, ctx, neg = _klein(monkeypatch)
    model = Flux2Transformer(w, v, CPU)
    call = lambda **kw: sampling.denoise(model, kw.pop("noise", noise), kw.pop("text", ctx),
                                         kw.pop("image_ids", image_ids), kw.pop("text_ids", text_ids), **kw)
    with pytest.raises(ValueError, match="Klein noise requires"):
        call(noise=noise[..., :8])
    with pytest.raises(ValueError, match="Klein text requires"):
        call(text=ctx[..., :8])
    with pytest.raises(ValueError, match="positions must match"):
        call(image_ids=image_ids[:, :5])
    with pytest.raises(ValueError, match="supplied together"):
        call(references=noise)
    with pytest.raises(ValueError, match="incompatible shapes"):
        call(references=noise[..., :8], reference_ids=image_ids)
    with pytest.raises(ValueError, match="explicit negative embeddings"):
        call(recipe=SamplingRecipe(variant="base"))
    with pytest.raises(ValueError, match="require active CFG"):
        call(negative=neg)
    with pytest.raises(ValueError, match="common FP16, BF16, or FP32"):
        call(text=ctx.double())
    bad = noise.clone()
    bad[0, 0, 0] = float("inf")
    with pytest.raises(ValueError, match="must be finite"):
        call(noise=bad)


# ----------------------------------------------------------------------------- LTX-2 states
def _ltx(monkeypatch):
    stand_in.install(monkeypatch)
    v = LTXVariant(dim=256, heads=2, context_dim=256, blocks=2)
    w = _kaiming(ltx_weights(v, seed=150, dtype=F32))
    latent = normal((1, 2 * 3 * 4, v.in_channels), seed=151, dtype=F32)
    context = normal((1, 6, v.context_dim), seed=152, dtype=F32)
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 4))
    return v, w, latent, context, pos


def test_ltx_denoise_loop_on_states_matches_oracle(monkeypatch):
    v, w, latent, context, pos = _ltx(monkeypatch)
    model = LTXVideoTransformer(w, v, CPU)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = lref.denoise(w, latent, context, pos, sigmas, v)
    state = ldn.LatentState(latent=latent.clone(), denoise_mask=torch.ones(1, latent.shape[1]),
                            positions=pos, clean_latent=latent.clone())
    ticks = []
    video, audio = ldn.denoise_loop(state, None, sigmas, transformer=model, video_context=context,
                                    callback=lambda i, n: ticks.append((i, n)))
    assert audio is None and torch.equal(state.latent, latent)  # the input state is untouched
    assert _max_rel(video.latent - latent, expect - latent) < TOL
    assert ticks == [(1, 3), (2, 3), (3, 3)] and video.positions is pos
    one, _ = ldn.denoise_step(state, None, sigma=sigmas[0], sigma_next=sigmas[1], transformer=model,
                              video_context=context)
    first = lref.denoise(w, latent, context, pos, sigmas[:2], v)
    assert _max_rel(one.latent - latent, first - latent) < TOL


def test_ltx_denoise_refusals_and_nonfinite_step(monkeypatch):
    v, w, latent, context, pos = _ltx(monkeypatch)
    model = LTXVideoTransformer(w, v, CPU)
    state = ldn.LatentState(latent=latent, denoise_mask=None, positions=pos)
    loop = lambda sig, **kw: ldn.denoise_loop(kw.pop("state", state), None, sig, transformer=model,
                                              video_context=context, **kw)
    with pytest.raises(ValueError, match="at least two sigmas"):
        loop((1.0,))
    with pytest.raises(ValueError, match="strictly descending"):
        loop((0.9, 0.9, 0.0))
    with pytest.raises(ValueError, match="positive and finite"):
        loop((0.9, 0.0, 0.0))
    with pytest.raises(ValueError, match="needs the stage"):
        loop((0.9, 0.0), step_kind="ancestral-rf")
    with pytest.raises(ValueError, match="deterministic Euler step only"):
        loop((0.9, 0.0), step_kind="ancestral-rf", stage=1)
    with pytest.raises(ValueError, match="uniform video denoise masks"):
        loop((0.9, 0.0), state=ldn.LatentState(latent, torch.ones(1, 24), pos, latent, False))
    with pytest.raises(ValueError, match="audio text mask needs an audio latent state"):
        loop((0.9, 0.0), audio_context_mask=torch.ones(1, 6))
    with pytest.raises(ValueError, match="per-query masks"):
        loop((0.9, 0.0), video_context_mask=torch.ones(1, 3, 6))
    with pytest.raises(ValueError, match="audio context is required"):
        ldn.denoise_step(state, state, sigma=0.9, sigma_next=0.5, transformer=model,
                         video_context=context)
    run, calls = model.run, []

    def poisoned(*args, **kwargs):
        out = run(*args, **kwargs)
        calls.append(1)
        if len(calls) == 2:
            out.fill_(float("nan"))
        return out

    monkeypatch.setattr(model, "run", poisoned)
    with pytest.raises(ldn.LTX2DenoiseError, match=r"stage 1, step 2: LTX-2 denoising produced a "
                                                   r"nonfinite video latent"):
        loop((0.9, 0.7, 0.5, 0.0), stage=1)


# ----------------------------------------------------------------------------- op contracts
def test_winograd_conv3d_and_euler_contracts():
    with pytest.raises(ValueError, match="positive multiple of four"):
        WinogradConv3d(transient_output_block=6)
    conv = WinogradConv3d(transient_output_block=8)
    x = torch.zeros((1, 3, 4, 5, 64), dtype=torch.bfloat16)
    w = torch.zeros((64, 3, 3, 3, 64), dtype=torch.bfloat16)
    assert not WinogradConv3d.supports(x, w)  # host tensors: the device conv does not take them
    assert not WinogradConv3d.supports(x[0], w)
    with pytest.raises(ValueError, match="batch-one BTHWC and OTHWI"):
        conv(x, w[:, :2], torch.zeros(64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="batch-one BTHWC and OTHWI"):
        conv(x, w.float(), torch.zeros(64))
    s = torch.zeros((4, 8))
    with pytest.raises(ValueError, match="positive and finite"):
        steps.euler_step(s, s, 0.0, 0.0)
    with pytest.raises(ValueError, match="must be finite"):
        steps.euler_velocity_step(s, s, float("nan"), 0.0)
    with pytest.raises(ValueError, match="does not match sample"):
        steps.euler_velocity_step(s, s[:2], 1.0, 0.5)
    with pytest.raises(ValueError, match="dtype"):
        steps.euler_velocity_step(s, s.double(), 1.0, 0.5)
