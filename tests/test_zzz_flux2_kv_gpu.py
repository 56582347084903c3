"""Device Klein KV editing and in-context references against the CPU oracle (oracle/flux2.py).

Collected after the other GPU tests, so that a failure here under `pytest -x` stops nothing else.

What each check can see, measured on the oracle (bf16 against fp32 on the same inputs; the
timestep is 500, which bf16 holds exactly: the reference rounds timestep x 1000 to the model
dtype, so a value bf16 cannot hold would give the two precisions different inputs):
  * with projection weights at std 1/sqrt(fan_in) (modulations x2, QK-norm weights perturbed
    off 1), the kept reference keys/values move by 0.5-0.7% (relative L2) under bf16 rounding,
    while reference rows on the current modulation move the second layer's keys by 72% and
    reference queries that also see text and target keys by 19%: gate 2e-2;
  * at the same weights the velocities of one extracting and one reusing evaluation move by
    0.7% under bf16 rounding, while leaving the reference out moves them by 7.7% and the
    reference rows on the current modulation by 3.6%: gate 2e-2 and cosine >= 0.999;
  * the kept rows depend on the reference rows alone, so two extractions with different
    targets, texts and timesteps keep bit-identical rows on the device (every kernel computes
    rows independently and deterministically);
  * whole trajectories at the synthetic weights (std 0.02): final-latent cosine >= 0.999 and
    relative L2 <= 3e-2, the gate of the other trajectory tests.

Seeds: weights S, target latents S + 1, text S + 2, references S + 3, all N(0, 1) on the CPU.
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as ref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import Flux2Transformer
from kinomlx_b200.synthetic import flux_weights, normal

pytestmark = pytest.mark.gpu
BF, F32 = torch.bfloat16, torch.float32
H, W, NR = 8, 12, 48  # a 96-token target grid and a 48-token (6 x 8) reference


def _variant(double: int = 1, single: int = 1) -> fcfg.FluxVariant:
    return fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072,
                            rope_axes=(32, 32, 32, 32), rope_theta=2000.0, in_channels=128,
                            context_dim=512, double_blocks=double, single_blocks=single)


def _scaled(w: dict, seed: int) -> dict:
    out = {}
    for name, t in w.items():
        if t.dim() == 2 and name.endswith(".weight") and "norm" not in name:
            t = t.float() / t.float().std() * t.shape[1] ** -0.5 * (2.0 if "modulation" in name else 1.0)
        elif t.dim() == 1 and "norm" in name:
            t = t.float() + 0.2 * normal(t.shape, seed=seed + len(out), dtype=F32)
        out[name] = t.to(BF)
    return out


def _case(seed: int, nt: int):
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    ref_ids = ref.image_ids(6, 8, 4)
    ref_ids[..., 0] = 10
    return dict(
        noise=normal((1, H * W, 128), seed=seed + 1),
        text=normal((1, nt, 512), seed=seed + 2),
        refs=normal((1, NR, 128), seed=seed + 3),
        text_ids=text_ids, image_ids=ref.image_ids(H, W, 4), ref_ids=ref_ids)


def _metrics(out: torch.Tensor, expect: torch.Tensor) -> tuple[float, float]:
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return float((o - e).norm() / e.norm()), float(torch.nn.functional.cosine_similarity(o, e, dim=0))


def _oracle_pair(w: dict, c: dict, v, t: float):
    """fp32 oracle on the bf16 values: extracting velocity, reusing velocity, kept rows."""
    w32 = {k: x.float() for k, x in w.items()}
    proj = ref.linear(c["text"].float(), w32["context_embedder.weight"])
    cx, sx = ref.rotary_positions(torch.cat([c["text_ids"], c["ref_ids"], c["image_ids"]], 1), v)
    cr, sr = ref.rotary_positions(torch.cat([c["text_ids"], c["image_ids"]], 1), v)
    state = ref.ReferenceKV(NR, v.double_blocks + v.single_blocks)
    tt = torch.tensor([t])
    image = torch.cat([c["refs"], c["noise"]], 1).float()
    extracting = ref.forward(w32, proj, cx, sx, image, tt, v, reference_kv=state)
    state.extracting = False
    reusing = ref.forward(w32, proj, cr, sr, c["noise"].float(), tt, v, reference_kv=state)
    return extracting, reusing, [state.tensors(i) for i in range(len(state.layers))]


def _device_pair(model: Flux2Transformer, c: dict, t: float, dev):
    extract, reuse = model.prepare_layouts(
        c["text"], (torch.cat([c["text_ids"], c["ref_ids"], c["image_ids"]], 1),
                    torch.cat([c["text_ids"], c["image_ids"]], 1)))
    cache = model.new_reference_kv(NR)
    image = torch.cat([c["refs"], c["noise"]], 1).to(dev)
    extracting = model.run(extract, image, t * 1000, reference_kv=cache).clone()
    cache.extracting = False
    reusing = model.run(reuse, c["noise"].to(dev), t * 1000, reference_kv=cache).clone()
    kept = [tuple(x.clone() for x in cache.tensors(i)) for i in range(cache.layer_count)]
    cache.clear()
    return extracting, reusing, kept


@pytest.mark.parametrize("nt", [40, 256])
def test_kept_reference_rows_match_oracle(cuda_device, nt):
    """Split (40 text rows) and joint (256) double-block paths: every layer's kept keys and
    values against the oracle's at weights where a mis-wired reference row shows."""
    v = _variant()
    w = _scaled(flux_weights(v, seed=31, dtype=F32), 31)
    c = _case(31, nt)
    _, _, kept = _oracle_pair(w, c, v, 0.5)
    _, _, got = _device_pair(Flux2Transformer(w, v, cuda_device), c, 0.5, cuda_device)
    torch.cuda.synchronize()
    for layer, ((ek, ev), (gk, gv)) in enumerate(zip(kept, got)):
        for name, e, g in (("key", ek, gk), ("value", ev, gv)):
            rel, cos = _metrics(g, e)
            assert rel <= 2e-2, (layer, name, rel, cos)


def test_kept_rows_depend_on_the_reference_alone(cuda_device):
    """Two extractions with other targets, texts and timesteps keep bit-identical rows."""
    v = _variant(2, 2)
    w = flux_weights(v, seed=51)
    model = Flux2Transformer(w, v, cuda_device)
    a, b = _case(51, 40), _case(61, 40)
    b["refs"] = a["refs"]
    _, _, kept_a = _device_pair(model, a, 0.5, cuda_device)
    _, _, kept_b = _device_pair(model, b, 0.25, cuda_device)
    torch.cuda.synchronize()
    for (ka, va), (kb, vb) in zip(kept_a, kept_b):
        assert torch.equal(ka, kb) and torch.equal(va, vb)


@pytest.mark.parametrize("nt", [40, 256])
def test_extracting_and_reusing_velocities_match_oracle(cuda_device, nt):
    v = _variant()
    w = _scaled(flux_weights(v, seed=21, dtype=F32), 21)
    c = _case(21, nt)
    ex, ru, _ = _oracle_pair(w, c, v, 0.5)
    gx, gr, _ = _device_pair(Flux2Transformer(w, v, cuda_device), c, 0.5, cuda_device)
    torch.cuda.synchronize()
    for name, g, e in (("extracting", gx, ex), ("reusing", gr, ru)):
        rel, cos = _metrics(g, e)
        assert rel <= 2e-2 and cos >= 0.999, (name, rel, cos)


@pytest.mark.parametrize("recompute", [False, True])
def test_kv_trajectory_matches_oracle(cuda_device, recompute):
    v = _variant()
    w = flux_weights(v, seed=71)
    c = _case(71, 40)
    sigmas = ref.schedule(H * W, 3)
    expect = ref.denoise_kv(w, c["noise"], c["text"], c["text_ids"], c["image_ids"], c["refs"],
                            c["ref_ids"], sigmas, v, recompute=recompute)
    model = Flux2Transformer(w, v, cuda_device)
    out = sampling.denoise_kv(model, c["noise"], c["text"], c["text_ids"], c["image_ids"],
                              c["refs"], c["ref_ids"], sigmas=sampling.schedule(H * W, 3),
                              recompute_reference_kv=recompute)
    rel, cos = _metrics(out, expect)
    assert out.shape == c["noise"].shape and cos >= 0.999 and rel <= 3e-2, (rel, cos)


def test_in_context_reference_trajectory_matches_oracle(cuda_device):
    """References appended after the target rows (the non-KV variants): only target rows move."""
    v = _variant()
    w = flux_weights(v, seed=81)
    c = _case(81, 40)
    ids = torch.cat([c["text_ids"], c["image_ids"], c["ref_ids"]], 1)
    sigmas = ref.schedule(H * W, 3)
    expect = ref.denoise(w, c["noise"], c["text"], ids, sigmas, v, references=c["refs"])
    model = Flux2Transformer(w, v, cuda_device)
    out = sampling.denoise_joint(model, c["noise"], c["text"], ids, sigmas=sampling.schedule(H * W, 3),
                           references=c["refs"])
    rel, cos = _metrics(out, expect)
    assert out.shape == c["noise"].shape and cos >= 0.999 and rel <= 3e-2, (rel, cos)


def test_reference_attention_function_matches_oracle(cuda_device):
    """The reference-shaped function on the reference test's geometry (2 text, 3 reference, 4
    target rows; here 128-wide heads and bf16): extraction against the fp32 oracle, reuse on the
    active rows against the extraction's rows."""
    from kinomlx_b200.flux2.kv import ReferenceKV, reference_attention

    q, k, v = (normal((1, 9, 2, 128), seed=90 + i) for i in range(3))
    expect = ref.reference_attention(q.float(), k.float(), v.float(), text_tokens=2,
                                     state=ref.ReferenceKV(3, 1), layer=0)
    state = ReferenceKV(3, 1, 1, 256, cuda_device, BF)
    out = reference_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                              text_tokens=2, state=state, layer=0)
    rel, cos = _metrics(out, expect)
    assert out.shape == q.shape and rel <= 1e-2 and cos >= 0.9999, (rel, cos)
    state.extracting = False
    active = torch.tensor([0, 1, 5, 6, 7, 8])
    again = reference_attention(q[:, active].to(cuda_device), k[:, active].to(cuda_device),
                                v[:, active].to(cuda_device), text_tokens=2, state=state, layer=0)
    rel, cos = _metrics(again, out[:, active.to(cuda_device)])
    assert rel <= 1e-2, (rel, cos)
