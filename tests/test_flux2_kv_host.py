"""Host logic of the device reference paths on the CPU (kernel calls replaced by the torch
stand-ins of tests/stand_in_kernels.py): for KV editing, the cache's lifetime when the loop fails
or is interrupted, the extraction/reuse sequence the loop drives, and the refusals of
`Flux2Transformer.run` and `sampling.denoise_kv`, which follow the reference's
(kinomlx/models/flux2/transformer.py:321-332, sampling.py:133-165, kv.py:30-45); for in-context
references, the reference sampling test's known answer (tests/models/flux2/test_sampling.py:
150-169) and its refusal of references without positions."""

from __future__ import annotations

import pytest
import torch

import stand_in_kernels as stand_in
from oracle import flux2 as fref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.kv import ReferenceKV
from kinomlx_b200.flux2.transformer import Flux2Transformer
from kinomlx_b200.synthetic import flux_weights, normal

F32 = torch.float32
CPU = torch.device("cpu")
V = fcfg.FluxVariant(dim=256, heads=2, mlp="swiglu", mlp_hidden=512, rope_axes=(32, 32, 32, 32),
                     rope_theta=2000.0, in_channels=32, context_dim=64, double_blocks=1,
                     single_blocks=1)


def _case(nt=8, h=2, w=3, nr=4):
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    ref_ids = fref.image_ids(2, 2, 4)
    ref_ids[..., 0] = 10
    return dict(noise=normal((1, h * w, 32), seed=1, dtype=F32), text=normal((1, nt, 64), seed=2, dtype=F32),
                text_ids=text_ids, image_ids=fref.image_ids(h, w, 4),
                references=normal((1, nr, 32), seed=3, dtype=F32), reference_ids=ref_ids)


class _Recording(Flux2Transformer):
    """Records (rows, extracting) per evaluation and can fail at evaluation `fail_at`."""

    def __init__(self, *args, fail=None, fail_at=0, **kw):
        super().__init__(*args, **kw)
        self.calls, self.caches, self.fail, self.fail_at = [], [], fail, fail_at

    def new_reference_kv(self, reference_tokens, batch=1):
        cache = super().new_reference_kv(reference_tokens, batch)
        self.caches.append(cache)
        return cache

    def run(self, prepared, image, t, **kw):
        kv = kw.get("reference_kv")
        self.calls.append((image.shape[1], None if kv is None else kv.extracting))
        if self.fail is not None and len(self.calls) == self.fail_at:
            raise self.fail("denoise interrupted")
        return super().run(prepared, image, t, **kw)


def _run(model, steps=3, recompute=False):
    c = _case()
    return sampling.denoise_kv(model, c["noise"], c["text"], c["text_ids"], c["image_ids"],
                               c["references"], c["reference_ids"],
                               sigmas=sampling.linear_sigmas(steps), recompute_reference_kv=recompute)


@pytest.mark.parametrize("recompute", [False, True])
def test_extraction_then_reuse_and_the_cache_is_released(monkeypatch, recompute):
    stand_in.install(monkeypatch)
    model = _Recording(flux_weights(V, seed=4, dtype=F32), V, CPU)
    _run(model, 3, recompute)
    extracting = [(4 + 6, True)]
    assert model.calls == (extracting * 3 if recompute else extracting + [(6, False)] * 2)
    assert len(model.caches) == (3 if recompute else 1)
    assert all(c.closed for c in model.caches)


@pytest.mark.parametrize("error", [RuntimeError, KeyboardInterrupt])
@pytest.mark.parametrize("step", [1, 2])
def test_failure_and_cancellation_release_the_cache(monkeypatch, error, step):
    stand_in.install(monkeypatch)
    model = _Recording(flux_weights(V, seed=4, dtype=F32), V, CPU, fail=error, fail_at=step)
    with pytest.raises(error):
        _run(model)
    assert model.caches[0].closed
    with pytest.raises(ValueError, match="not been extracted"):
        model.caches[0].tensors(0)


def test_run_refuses_what_the_reference_refuses(monkeypatch):
    stand_in.install(monkeypatch)
    model = Flux2Transformer(flux_weights(V, seed=4, dtype=F32), V, CPU)
    c = _case()
    extract, _ = model.prepare_layouts(c["text"], (
        torch.cat([c["text_ids"], c["reference_ids"], c["image_ids"]], 1),
        torch.cat([c["text_ids"], c["image_ids"]], 1)))
    image = torch.cat([c["references"], c["noise"]], 1)
    closed = model.new_reference_kv(4)
    closed.clear()
    with pytest.raises(ValueError, match="completed generation"):
        model.run(extract, image, 500.0, reference_kv=closed)
    with pytest.raises(ValueError, match="layer count"):
        model.run(extract, image, 500.0, reference_kv=ReferenceKV(4, 3, 1, V.dim, CPU, F32))
    with pytest.raises(ValueError, match="batch"):
        model.run(extract, image, 500.0, reference_kv=model.new_reference_kv(4, batch=2))
    with pytest.raises(ValueError, match="followed by target tokens"):
        model.run(extract, c["references"], 500.0, reference_kv=model.new_reference_kv(4))
    with pytest.raises(ValueError, match="positive token and layer counts"):
        model.new_reference_kv(0)
    with pytest.raises(ValueError, match="outside"):
        model.run(extract, image, 500.0, target=(8, 4))


def test_denoise_kv_refuses_mismatched_inputs(monkeypatch):
    stand_in.install(monkeypatch)
    model = Flux2Transformer(flux_weights(V, seed=4, dtype=F32), V, CPU)
    c = _case()
    sig = sampling.linear_sigmas(2)
    args = lambda **o: {**c, **o}
    call = lambda a: sampling.denoise_kv(model, a["noise"], a["text"], a["text_ids"], a["image_ids"],
                                         a["references"], a["reference_ids"], sigmas=sig)
    with pytest.raises(ValueError, match="incompatible shapes"):
        call(args(reference_ids=c["reference_ids"][:, :3]))
    with pytest.raises(ValueError, match="incompatible shapes"):
        call(args(references=normal((1, 4, 16), seed=5, dtype=F32)))
    with pytest.raises(ValueError, match="positions must match"):
        call(args(image_ids=c["image_ids"][:, :5]))
    with pytest.raises(ValueError, match="no reference K/V path"):
        sampling.denoise_kv(object(), c["noise"], c["text"], c["text_ids"], c["image_ids"],
                            c["references"], c["reference_ids"], sigmas=sig)


def test_reference_attention_function_matches_oracle(monkeypatch):
    """The reference-shaped function on the reference test's geometry (9 rows: 2 text, 3
    reference, 4 target) with 128-wide heads: extraction against the oracle, reuse on the active
    rows against the extraction's rows."""
    from kinomlx_b200.flux2.kv import reference_attention

    stand_in.install(monkeypatch)
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn((1, 9, 2, 128), generator=g) for _ in range(3))
    expect = fref.reference_attention(q, k, v, text_tokens=2, state=fref.ReferenceKV(3, 1), layer=0)
    state = ReferenceKV(3, 1, 1, 256, CPU, F32)
    out = reference_attention(q, k, v, text_tokens=2, state=state, layer=0)
    assert out.shape == q.shape and float((out - expect).abs().max()) < 1e-5
    state.extracting = False
    active = torch.tensor([0, 1, 5, 6, 7, 8])
    again = reference_attention(q[:, active], k[:, active], v[:, active], text_tokens=2, state=state, layer=0)
    assert float((again - out[:, active]).abs().max()) < 1e-5


class _TextVelocity:
    """The reference sampling test's stand-in model (tests/models/flux2/test_sampling.py:136-142):
    every row's velocity is the first value of its batch entry's text; it records each image it
    is given. Runs the `Flux2Transformer.run` contract (fused Euler, target rows)."""

    device, dtype = CPU, F32

    def __init__(self):
        from kinomlx_b200.sequence_parallel import SequenceParallel

        self.sp = SequenceParallel.single()
        self.inputs = []

    def prepare(self, text, ids):
        return text

    def run(self, prepared, image, t, *, euler_dt=None, sample=None, out=None, target=None):
        self.inputs.append(image.clone())
        first, rows = target or (0, image.shape[1])
        velocity = torch.ones_like(image[:, first : first + rows]) * prepared[:, :1, :1]
        if euler_dt is None:
            return velocity
        out.copy_(sample + euler_dt * velocity)
        return out


@pytest.mark.parametrize("guidance", [1.0, 4.0])
def test_cfg_updates_only_targets_and_keeps_references_fixed(monkeypatch, guidance):
    """The reference's known answer: with negative = -text and guidance 4 the combined velocity
    is -1 + 4 * 2 = 7, so a schedule from 1 to 0 ends at -7 (at guidance 1, -1); the reference
    rows every evaluation sees stay 17."""
    stand_in.install(monkeypatch)
    model = _TextVelocity()
    noise, text = torch.zeros((1, 4, 32)), torch.ones((1, 2, 64))
    ids = torch.zeros((1, 2 + 4 + 3, 4), dtype=torch.int64)
    result = sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.schedule(4, 4),
                              negative=-text if guidance != 1.0 else None, guidance=guidance,
                              references=torch.full((1, 3, 32), 17.0))
    assert result.shape == noise.shape
    assert float((result + (7.0 if guidance != 1.0 else 1.0)).abs().max()) < 1e-6
    assert len(model.inputs) == 4 and all(bool((seen[:, 4:] == 17).all()) for seen in model.inputs)


def test_references_without_their_positions_fail_before_any_evaluation(monkeypatch):
    stand_in.install(monkeypatch)
    model = _TextVelocity()
    with pytest.raises(ValueError, match="positions must match"):
        sampling.denoise_joint(model, torch.zeros((1, 4, 32)), torch.ones((1, 2, 64)),
                         torch.zeros((1, 6, 4), dtype=torch.int64), sigmas=sampling.schedule(4, 4),
                         references=torch.zeros((1, 1, 32)))
    assert not model.inputs
