"""Device Flux2 MMDiT against the CPU oracle on identical seeded inputs.

Gates (BASELINE): per-op max relative error <= 2e-2 in bf16 (tests/test_gpu_kernels.py) and
final-latent cosine similarity >= 0.999 after the full step schedule. Block outputs are also
held to a relative L2 error <= 1e-2.

Seeds and draw order: weights from seed S (kinomlx_b200.synthetic order), image hidden/latent
from S + 1, text from S + 2, negative text from S + 3, all N(0, 1), drawn on the CPU.
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as ref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import Flux2Transformer, rotary_positions
from kinomlx_b200.synthetic import flux_weights, normal

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _metrics(out: torch.Tensor, expect: torch.Tensor) -> tuple[float, float, float]:
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    rel_l2 = float((o - e).norm() / e.norm())
    max_rel = float((o - e).abs().max() / e.abs().max())
    cos = float(torch.nn.functional.cosine_similarity(o, e, dim=0))
    return rel_l2, max_rel, cos


def _ids(h: int, w: int, text: int, axes: int = 2) -> torch.Tensor:
    return torch.cat([torch.zeros((1, text, axes), dtype=torch.int64), ref.image_ids(h, w, axes)], 1)


def test_config1_double_block_matches_oracle(cuda_device):
    """one MMDiT double block, 512 text + 1024 image tokens, hidden 3072,
    24 heads, t = 0.5, seed 0, bf16."""
    v = fcfg.BASELINE.with_blocks(1, 0)
    w = flux_weights(v, seed=0)
    image = normal((1, 1024, v.dim), seed=1)
    text = normal((1, 512, v.dim), seed=2)
    ids = _ids(32, 32, 512)
    t = torch.tensor([0.5], dtype=BF)

    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    im = ref.modulation(w, "double_stream_modulation_img", emb)
    tm = ref.modulation(w, "double_stream_modulation_txt", emb)
    exp_img, exp_txt = ref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)

    model = Flux2Transformer(w, v, cuda_device)
    cos, sin = rotary_positions(ids, v)
    t_dev = (t * 1000).float().to(cuda_device)
    img, txt = model.double_block(0, image.to(cuda_device), text.to(cuda_device), t_dev,
                                  cos.to(cuda_device), sin.to(cuda_device))
    for out, exp in ((img, exp_img), (txt, exp_txt)):
        rel_l2, max_rel, cosine = _metrics(out, exp)
        assert rel_l2 <= 1e-2, rel_l2
        assert max_rel <= 2e-2, max_rel
        assert cosine >= 0.999, cosine


def test_single_block_matches_oracle(cuda_device):
    v = fcfg.BASELINE.with_blocks(0, 1)
    w = flux_weights(v, seed=5)
    nt, h, wd = 128, 16, 24
    value = normal((1, nt + h * wd, v.dim), seed=6)
    ids = _ids(h, wd, nt)
    t = torch.tensor([0.75], dtype=BF)
    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    sm = ref.modulation(w, "single_stream_modulation", emb)
    expect = ref.single_block(w, 0, value, sm, cos4, sin4, v)
    model = Flux2Transformer(w, v, cuda_device)
    cos, sin = rotary_positions(ids, v)
    out = model.single_block(0, value.to(cuda_device), nt, (t * 1000).float().to(cuda_device),
                             cos.to(cuda_device), sin.to(cuda_device))
    rel_l2, max_rel, cosine = _metrics(out, expect)
    assert rel_l2 <= 1e-2 and max_rel <= 2e-2 and cosine >= 0.999, (rel_l2, max_rel, cosine)


@pytest.mark.parametrize("cfg", [False, True])
def test_denoise_schedule_matches_oracle(cuda_device, cfg):
    """A 2 double + 2 single block model over a 3-step linear schedule (4 with CFG off):
    final-latent cosine >= 0.999 against the oracle's trajectory."""
    v = fcfg.BASELINE.with_blocks(2, 2)
    w = flux_weights(v, seed=42)
    h, wd, nt = 16, 16, 64
    noise = normal((1, h * wd, v.in_channels), seed=43)
    text = normal((1, nt, v.context_dim), seed=44)
    negative = normal((1, nt, v.context_dim), seed=45) if cfg else None
    ids = _ids(h, wd, nt)
    steps = 3 if cfg else 4
    sigmas = ref.linear_sigmas(steps)
    expect = ref.denoise(w, noise, text, ids, sigmas, v, negative=negative,
                         guidance=4.0 if cfg else 1.0)
    model = Flux2Transformer(w, v, cuda_device)
    out = sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.linear_sigmas(steps),
                           negative=negative, guidance=4.0 if cfg else 1.0)
    rel_l2, max_rel, cosine = _metrics(out, expect)
    assert cosine >= 0.999, (rel_l2, max_rel, cosine)
    assert rel_l2 <= 3e-2, (rel_l2, max_rel, cosine)


def test_full_size_step_is_finite(cuda_device):
    """BASELINE config 2 shapes (4096 image + 512 text tokens, 8 + 24 blocks), weights drawn on
    the GPU: one fused-Euler step runs and stays finite; deterministic across two runs."""
    v = fcfg.BASELINE
    w = flux_weights(v, seed=42, device=cuda_device)
    model = Flux2Transformer(w, v, cuda_device)
    noise = normal((1, 4096, v.in_channels), seed=43, device=cuda_device)
    text = normal((1, 512, v.context_dim), seed=44, device=cuda_device)
    ids = _ids(64, 64, 512)
    sig = sampling.linear_sigmas(4)
    prepared = model.prepare(text, ids)
    a = noise.clone()
    b = noise.clone()
    sampling.denoise_step(model, prepared, a, sig, 0)
    sampling.denoise_step(model, prepared, b, sig, 0)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(a).all())
    assert torch.equal(a, b)
    assert float((a.float() - noise.float()).abs().max()) > 0


def test_klein_swiglu_variant_matches_oracle(cuda_device):
    """The reference's own Klein graph shape (SwiGLU MLP with gate first, 4 interleaved-pair RoPE
    axes of 32 dims, theta 2000, 128-channel latents), narrowed to hidden 1024 / 8 heads so the
    oracle stays quick: a 2-step trajectory, final-latent cosine >= 0.999."""
    v = fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072,
                         rope_axes=(32, 32, 32, 32), rope_theta=2000.0, in_channels=128,
                         context_dim=512, double_blocks=1, single_blocks=1)
    w = flux_weights(v, seed=21)
    h, wd, nt = 8, 12, 40
    noise = normal((1, h * wd, v.in_channels), seed=22)
    text = normal((1, nt, v.context_dim), seed=23)
    img = torch.zeros((1, h * wd, 4), dtype=torch.int64)
    img[0, :, 1] = torch.arange(h).repeat_interleave(wd)
    img[0, :, 2] = torch.arange(wd).repeat(h)
    txt = torch.zeros((1, nt, 4), dtype=torch.int64)
    txt[0, :, 3] = torch.arange(nt)
    ids = torch.cat([txt, img], 1)
    sigmas = ref.schedule(h * wd, 2)
    expect = ref.denoise(w, noise, text, ids, sigmas, v)
    model = Flux2Transformer(w, v, cuda_device)
    out = sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.schedule(h * wd, 2))
    rel_l2, max_rel, cosine = _metrics(out, expect)
    assert cosine >= 0.999 and rel_l2 <= 3e-2, (rel_l2, max_rel, cosine)
