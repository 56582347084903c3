"""Parity at BASELINE's own sizes: the device path against the CPU oracle on identical seeded
inputs, at the exact shapes of configs 2, 4 and 5.

- config 2: the full image DiT (4096 image + 512 text tokens, hidden 3072, 8 double + 24 single
  blocks, GELU MLP x4, 2D axial RoPE): the velocity of the first evaluation, and the whole
  4-step linear-sigma Euler schedule (gate: final-latent cosine >= 0.999, BASELINE's bar, and
  the same bars on the update final - noise, which the noise does not dominate);
- config 4: one full-width LTX-2 video block at 9216 video + 256 text tokens (width 4096,
  32 heads), the velocity and its X0 + Euler step; the block's own contribution is checked
  against the oracle's zero-block velocity as well;
- config 5: one full-width VAE decoder tile (8 x 8 latent, 16 frames, widths
  1024 -> 512 -> 256 -> 128, GroupNorm(32) + SiLU, causal convs) to its 3 x 121 x 256 x 256
  output, with conv biases and GroupNorm affines moved off their 0 / 1 defaults so every
  term is exercised.

Per-op bars of BASELINE: max relative error <= 2e-2 in bf16, here read both as max |o - e| /
max |e| and as the elementwise relative error of every value above a tenth of the tensor's
rms (see parity_metrics). The oracle rounds to bf16 at the reference's rounding points and
accumulates in fp32, as the device does, so what remains is accumulation order and the
device's exp2 / rsqrt.

The CPU oracle takes minutes at these sizes (about 40 s per config-2 evaluation on 16 host
cores), so this file runs after the other GPU tests; the weights are drawn on the CPU, in the
documented order, and copied to the device so both sides see the same bytes.
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as ref
from oracle import ltx2 as lref
from oracle import video_vae as vref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import Flux2Transformer
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2 import video_vae as vae
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.synthetic import flux_weights, ltx_weights, make_weights, normal
from parity_metrics import metrics, show, update_metrics

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _check(name: str, m: dict[str, float], *, rel_l2: float, max_norm: float, cos: float,
           elem_p999: float | None = None) -> None:
    print(show(name, m))
    assert m["rel_l2"] <= rel_l2, show(name, m)
    assert m["max_norm"] <= max_norm, show(name, m)
    assert m["cos"] >= cos, show(name, m)
    if elem_p999 is not None:
        assert m["elem_p999"] <= elem_p999, show(name, m)


# ----------------------------------------------------------------------------- config 2
@pytest.fixture(scope="module")
def config2():
    """Seeds as bench.py's config 2: weights 42, latent 43, text 44 (text width 4096)."""
    v = fcfg.BASELINE
    w = flux_weights(v, seed=42)
    noise = normal((1, 4096, v.in_channels), seed=43)
    text = normal((1, 512, v.context_dim), seed=44)
    ids = torch.cat([torch.zeros((1, 512, 2), dtype=torch.int64), ref.image_ids(64, 64, 2)], 1)
    return v, w, noise, text, ids


def test_config2_first_velocity_full_size(cuda_device, config2):
    """The first evaluation's velocity against the bf16 oracle and against the same oracle in
    fp32 on the same bf16 weights and inputs. Through 32 blocks bf16 rounding alone moves the
    velocity: the bf16 oracle lies 1.52 % (relative L2) from the fp32 one, so the gate on the
    device is 2.5e-2 against either; the per-op bar (max relative error 2e-2) still holds."""
    v, w, noise, text, ids = config2
    sigmas = ref.linear_sigmas(4)
    t = ref.step_timestep(sigmas, 0, BF)
    projected, cos, sin = ref.prepare(w, text, ids, v)
    expect = ref.forward(w, projected, cos, sin, noise, t, v)
    w32 = {name: x.float() for name, x in w.items()}
    projected32, _, _ = ref.prepare(w32, text.float(), ids, v)
    exact = ref.forward(w32, projected32, cos, sin, noise.float(), t.float(), v)
    print(show("bf16 oracle vs fp32 oracle", metrics(expect, exact)))

    model = Flux2Transformer(w, v, cuda_device)
    prepared = model.prepare(text.to(cuda_device), ids)
    got = model.run(prepared, noise.to(cuda_device),
                    float(sampling.timestep_x1000(sampling.linear_sigmas(4), 0))).clone()
    torch.cuda.synchronize()
    _check("config 2 velocity (32 blocks, 4608 tokens)", metrics(got, expect),
           rel_l2=2.5e-2, max_norm=2e-2, cos=0.9995)
    _check("config 2 velocity against the fp32 oracle", metrics(got, exact),
           rel_l2=2.5e-2, max_norm=2e-2, cos=0.9995)


def test_config2_full_schedule(cuda_device, config2):
    """All four Euler steps of config 2 (sigmas linspace(1, 0, 5), no CFG)."""
    v, w, noise, text, ids = config2
    expect = ref.denoise(w, noise, text, ids, ref.linear_sigmas(4), v)
    model = Flux2Transformer(w, v, cuda_device)
    got = sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.linear_sigmas(4))
    torch.cuda.synchronize()
    final = metrics(got, expect)
    print(show("config 2 final latent", final))
    assert final["cos"] >= 0.999, show("final", final)
    _check("config 2 update (final - noise)", update_metrics(got, expect, noise),
           rel_l2=2e-2, max_norm=2e-2, cos=0.999)


# ----------------------------------------------------------------------------- config 4
def test_config4_block_full_size(cuda_device):
    """One LTX-2 video block at 16 x 18 x 32 = 9216 video tokens and 256 text tokens."""
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=0)
    grid = (16, 18, 32)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=1)
    context = normal((1, 256, v.context_dim), seed=2)
    pos = lref.pixel_coords(lref.patch_grid_bounds(*grid))
    sigma, sigma_next = lref.DISTILLED_STAGE_1_SIGMAS[5], lref.DISTILLED_STAGE_1_SIGMAS[6]
    expect = lref.forward(w, latent, context, sigma, pos, v)
    before = lref.forward(w, latent, context, sigma, pos, v.with_blocks(0))
    expect_next = lref.euler_step(latent, lref.to_denoised(latent, sigma, expect), sigma, sigma_next)

    model = LTXVideoTransformer(w, v, cuda_device)
    prepared = model.prepare(context.to(cuda_device), pos)
    x = latent.to(cuda_device)
    got = model.run(prepared, x, sigma).clone()
    nxt = x.clone()
    model.run(prepared, nxt, sigma, sigma_next=sigma_next, out=nxt)
    torch.cuda.synchronize()
    _check("config 4 velocity (1 block, 9216 tokens)", metrics(got, expect),
           rel_l2=1e-2, max_norm=2e-2, cos=0.9999)
    _check("config 4 block contribution (velocity - zero-block velocity)",
           update_metrics(got, expect, before), rel_l2=3e-2, max_norm=5e-2, cos=0.999)
    # the next latent itself against the BASELINE bars; its update (next - latent) only on
    # rel-L2 and cosine: one bf16 ulp of a latent value near 3 is 2.4 % of the largest update
    _check("config 4 X0 + Euler next latent", metrics(nxt, expect_next),
           rel_l2=1e-2, max_norm=2e-2, cos=0.9999)
    m = update_metrics(nxt, expect_next, latent)
    print(show("config 4 X0 + Euler update", m))
    assert m["rel_l2"] <= 2e-2 and m["cos"] >= 0.999, show("config 4 update", m)


# ----------------------------------------------------------------------------- config 5
def test_config5_tile_full_width(cuda_device):
    """One 8 x 8-latent tile of config 5 through the whole decoder (16 latent frames ->
    121 frames of 256 x 256)."""
    v = vae.BASELINE_VAE
    rv = vref.BASELINE_VAE
    w = make_weights(vae.vae_weight_specs(v), seed=0)
    for i, name in enumerate(sorted(w)):  # biases and affines off their defaults
        if name.endswith(".bias") and "per_channel" not in name:
            w[name] = normal(w[name].shape, seed=1000 + i, std=0.05)
        elif name.endswith(".weight") and "norm" in name:
            w[name] = (1.0 + normal(w[name].shape, seed=1000 + i, dtype=torch.float32, std=0.2)).to(BF)
    latent = normal((1, 128, 16, 8, 8), seed=1)
    expect = vref.decode(w, latent, rv)
    dec = vae.VideoDecoder(w, v, cuda_device)
    got = dec.decode(latent.to(cuda_device), tile=None)
    torch.cuda.synchronize()
    assert tuple(got.shape) == tuple(expect.shape) == (1, 3, 121, 256, 256)
    _check("config 5 tile (1024 -> 128 channels, 121 x 256 x 256)", metrics(got, expect),
           rel_l2=2e-2, max_norm=2e-2, cos=0.999)
