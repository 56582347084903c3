"""Pins of the Klein KV-editing oracle (oracle/flux2.py: ReferenceKV, reference_attention,
blend_modulation, kv_loop, forward with reference K/V) against the reference's own tests
(tests/models/flux2/test_kv.py of KinoMLX): the dense-mask formula, cached recomputation,
independence of the reference rows, the modulation known answer, the extraction/reuse call
sequence and cache lifetime, and the reference's refusals. Plus two properties of the whole
model: the kept keys/values depend on the reference rows only, and recomputing the cache every
step gives the cached trajectory. CPU only."""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as fref
from kinomlx_b200.synthetic import flux_weights, normal

F32 = torch.float32


def _variant():
    return fref.FluxVariant(dim=256, heads=2, mlp="swiglu", mlp_hidden=512, rope_axes=(32, 32, 32, 32),
                            rope_theta=2000.0, in_channels=32, context_dim=64, double_blocks=1,
                            single_blocks=2)


def test_reference_attention_matches_dense_mask_and_cached_recomputation():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn((1, 9, 2, 8), generator=g) for _ in range(3))
    state = fref.ReferenceKV(3, 1)
    actual = fref.reference_attention(q, k, v, text_tokens=2, state=state, layer=0)
    scores = (q.transpose(1, 2) @ k.transpose(1, 2).transpose(-1, -2)) / 8 ** 0.5
    positions = torch.arange(9)
    reference = (positions >= 2) & (positions < 5)
    allowed = ~reference[:, None] | reference[None, :]
    expected = (torch.softmax(scores.masked_fill(~allowed, -torch.inf), -1) @ v.transpose(1, 2)).transpose(1, 2)
    assert float((actual - expected).abs().max()) < 1e-5
    state.extracting = False
    active = torch.tensor([0, 1, 5, 6, 7, 8])
    cached = fref.reference_attention(q[:, active], k[:, active], v[:, active], text_tokens=2,
                                      state=state, layer=0)
    assert float((cached - actual[:, active]).abs().max()) < 1e-5
    # reference outputs cannot depend on the current text or target tokens
    changed = torch.where(reference[None, :, None, None], v, v + 100)
    other = fref.reference_attention(q, k, changed, text_tokens=2, state=fref.ReferenceKV(3, 1), layer=0)
    assert torch.equal(other[:, 2:5], actual[:, 2:5])


def test_reference_modulation_only_replaces_reference_positions():
    current, fixed = torch.tensor([[1.0, 2.0]]), torch.tensor([[9.0, 10.0]])
    result = fref.blend_modulation(current, fixed, 2, 3, 7)
    assert result.tolist() == [
        [[1.0, 2.0], [1.0, 2.0], [9.0, 10.0], [9.0, 10.0], [9.0, 10.0], [1.0, 2.0], [1.0, 2.0]]
    ]


class _Recorder:
    """The reference test's stand-in model: extraction keeps the reference rows' first channel,
    every velocity is the kept rows' mean."""

    def __init__(self, fail=None, fail_at=2, scale=1.0):
        self.calls, self.caches = [], []
        self.fail, self.fail_at, self.scale = fail, fail_at, scale

    def new_cache(self, count):
        state = fref.ReferenceKV(count, 1)
        self.caches.append(state)
        return state

    def velocity(self, image, t, cache):
        self.calls.append((image.shape[1], cache.extracting))
        if cache.extracting:
            kept = image[:, : cache.reference_tokens, :1, None] * self.scale
            cache.store(0, kept, kept, 0, kept.shape[1])
            image = image[:, cache.reference_tokens :]
        if self.fail and len(self.calls) == self.fail_at:
            raise self.fail("denoise interrupted")
        return torch.ones_like(image) * cache.tensors(0)[0].mean()


def _loop(model, steps=4, recompute=False, reference_value=2.0):
    return fref.kv_loop(model.velocity, model.velocity, model.new_cache,
                        torch.full((1, 3, 8), reference_value), torch.zeros((1, 4, 8)),
                        fref.linear_sigmas(steps), recompute=recompute)


@pytest.mark.parametrize("steps", [1, 4])
def test_extraction_reuse_counts_and_repeated_generation_isolation(steps):
    model = _Recorder()
    first = _loop(model, steps)
    assert model.calls == [(7, True)] + [(4, False)] * (steps - 1)
    assert torch.equal(first, _loop(model, steps))
    model.scale = 3.0
    changed = _loop(model, steps)
    assert not torch.equal(first, changed)
    assert len({id(c) for c in model.caches}) == 3
    assert all(c.closed and c.layers[0] is None for c in model.caches)
    assert not torch.equal(changed, _loop(model, steps, reference_value=5.0))


def test_recomputation_gives_the_cached_result_with_an_extraction_per_step():
    cached = _loop(_Recorder())
    model = _Recorder()
    assert torch.equal(cached, _loop(model, recompute=True))
    assert model.calls == [(7, True)] * 4


@pytest.mark.parametrize("error", [RuntimeError, KeyboardInterrupt])
@pytest.mark.parametrize("step", [1, 2])
def test_failure_and_cancellation_clear_the_cache(error, step):
    model = _Recorder(fail=error, fail_at=step)
    with pytest.raises(error):
        _loop(model)
    assert model.caches[0].closed and model.caches[0].layers[0] is None


def _setup(nt=5, h=3, w=4, nr=6, seed=90):
    v = _variant()
    p = flux_weights(v, seed=seed, dtype=F32)
    text = normal((1, nt, v.context_dim), seed=seed + 1, dtype=F32)
    noise = normal((1, h * w, v.in_channels), seed=seed + 2, dtype=F32)
    refs = normal((1, nr, v.in_channels), seed=seed + 3, dtype=F32)
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    image_ids = fref.image_ids(h, w, 4)
    ref_ids = fref.image_ids(2, 3, 4)
    ref_ids[..., 0] = 10  # the reference's own time offset
    return v, p, text, noise, refs, text_ids, image_ids, ref_ids


def test_refusals_of_the_reference_forward():
    v, p, text, noise, refs, text_ids, image_ids, ref_ids = _setup()
    with pytest.raises(ValueError, match="positive token and layer counts"):
        fref.ReferenceKV(0, 3)
    projected = fref.linear(text, p["context_embedder.weight"])
    cos, sin = fref.rotary_positions(torch.cat([text_ids, ref_ids, image_ids], 1), v)
    t = torch.tensor([0.5])
    closed = fref.ReferenceKV(6, 3)
    closed.clear()
    with pytest.raises(ValueError, match="completed generation"):
        fref.forward(p, projected, cos, sin, torch.cat([refs, noise], 1), t, v, reference_kv=closed)
    with pytest.raises(ValueError, match="layer count"):
        fref.forward(p, projected, cos, sin, torch.cat([refs, noise], 1), t, v,
                     reference_kv=fref.ReferenceKV(6, 2))
    with pytest.raises(ValueError, match="followed by target tokens"):
        fref.forward(p, projected, cos[:, :11], sin[:, :11], refs, t, v,
                     reference_kv=fref.ReferenceKV(6, 3))
    with pytest.raises(ValueError, match="not been extracted"):
        fref.ReferenceKV(6, 3).tensors(0)


def test_kept_rows_depend_on_the_reference_only_and_recomputing_matches_reuse():
    """Reference rows see only reference keys and the timestep-0 modulation, so what a layer
    keeps is the same for any target, text or timestep; hence extracting at every step gives
    the trajectory of extracting once."""
    v, p, text, noise, refs, text_ids, image_ids, ref_ids = _setup()
    projected = fref.linear(text, p["context_embedder.weight"])
    cos, sin = fref.rotary_positions(torch.cat([text_ids, ref_ids, image_ids], 1), v)
    kept = []
    for seed, t in ((95, 0.8), (96, 0.3)):
        state = fref.ReferenceKV(refs.shape[1], 3)
        other = normal(noise.shape, seed=seed, dtype=F32)
        fref.forward(p, projected * (1 + seed % 2), cos, sin, torch.cat([refs, other], 1),
                     torch.tensor([t]), v, reference_kv=state)
        kept.append([state.tensors(i) for i in range(3)])
    for (k0, v0), (k1, v1) in zip(*kept):
        assert torch.allclose(k0, k1, atol=1e-6) and torch.allclose(v0, v1, atol=1e-6)
    sig = fref.linear_sigmas(3)
    once = fref.denoise_kv(p, noise, text, text_ids, image_ids, refs, ref_ids, sig, v)
    every = fref.denoise_kv(p, noise, text, text_ids, image_ids, refs, ref_ids, sig, v, recompute=True)
    assert float((once - every).abs().max()) < 1e-5 * float(once.abs().max())
