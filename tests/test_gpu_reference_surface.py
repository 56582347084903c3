"""The reference-signature call sites on the B200: the Euler steps of
kinomlx/samplers/steps.py:8-70 and kinomlx/models/flux2/sampling.py:109-113 bit-exact against
the oracle's formulas, `WinogradConv3d` against the oracle's conv, and the Klein / LTX-2 loops of
the reference's signatures against the bare device loops they wrap (the same launches, so the
same bits) and against each other where the reference offers two ways (batched and sequential
CFG; the Euler update fused into the final projection or, with `on_step`, as its own launch)."""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as ref
from oracle import ltx2 as lref
from oracle import video_vae as vref
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.sampling import SamplingRecipe
from kinomlx_b200.flux2.transformer import Flux2Transformer
from kinomlx_b200.kernels.winograd_conv3d import WinogradConv3d
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.samplers import steps
from kinomlx_b200.synthetic import flux_weights, ltx_weights, normal
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu
BF, F32 = torch.bfloat16, torch.float32


def test_euler_steps_bit_exact(cuda_device):
    x = normal((3, 1000, 8), seed=1)
    d = normal((3, 1000, 8), seed=2)
    sigma, nxt = 0.909375, 0.725
    # kinomlx/samplers/steps.py:36-70 in torch fp32 on the host, then rounded
    ratio = torch.tensor(nxt / sigma, dtype=F32)
    expect = (d.float() + ratio * (x.float() - d.float())).to(BF)
    got = steps.euler_step(x.to(cuda_device), d.to(cuda_device), sigma, nxt)
    assert torch.equal(got.cpu(), expect)
    got32 = steps.euler_step(x.float().to(cuda_device), d.float().to(cuda_device), sigma, nxt)
    assert torch.equal(got32.cpu(), d.float() + ratio * (x.float() - d.float()))
    # kinomlx/samplers/steps.py:8-33
    delta = torch.tensor(nxt - sigma, dtype=F32)
    expect = (x.float() + (delta * d.float()).to(BF).float()).to(BF)
    got = steps.euler_velocity_step(x.to(cuda_device), d.to(cuda_device), sigma, nxt)
    assert torch.equal(got.cpu(), expect)
    # kinomlx/models/flux2/sampling.py:109-113
    dt = torch.tensor(-0.25, dtype=F32)
    got = sampling.euler_step(x.to(cuda_device), d.to(cuda_device), dt)
    assert torch.equal(got.cpu(), ref.euler_step(x, d, dt))


@pytest.mark.parametrize("shape", [(5, 9, 11, 64, 128), (3, 16, 24, 128, 64)])
def test_winograd_conv3d_surface_matches_oracle(cuda_device, shape):
    f, h, w, cin, cout = shape
    x = normal((1, f, h, w, cin), seed=3)
    wt = normal((cout, 3, 3, 3, cin), seed=4, std=0.05)
    b = normal((cout,), seed=5, std=0.5)
    expect = vref.conv3d(x, wt, b, causal=False)
    conv = WinogradConv3d()
    dx, dw, db = x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device)
    assert conv.supports(dx, dw)
    got = conv(dx, dw, db)
    m = metrics(got, expect)
    assert tuple(got.shape) == tuple(expect.shape) and m["max_norm"] <= 2e-2, show("conv", m)


def _klein_case(cuda_device):
    v = fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072,
                         rope_axes=(32, 32, 32, 32), rope_theta=2000.0, in_channels=128,
                         context_dim=512, double_blocks=1, single_blocks=2)
    w = flux_weights(v, seed=31)
    h, wd, nt = 8, 12, 40
    noise = normal((1, h * wd, v.in_channels), seed=32)
    text = normal((1, nt, v.context_dim), seed=33)
    negative = normal((1, nt, v.context_dim), seed=34)
    image_ids = torch.zeros((1, h * wd, 4), dtype=torch.int64)
    image_ids[0, :, 1] = torch.arange(h).repeat_interleave(wd)
    image_ids[0, :, 2] = torch.arange(wd).repeat(h)
    text_ids = torch.zeros((1, nt, 4), dtype=torch.int64)
    text_ids[0, :, 3] = torch.arange(nt)
    return v, w, Flux2Transformer(w, v, cuda_device), noise, text, negative, image_ids, text_ids


def test_klein_denoise_reference_signature(cuda_device):
    v, w, model, noise, text, negative, image_ids, text_ids = _klein_case(cuda_device)
    sig = (1.0, 0.75, 0.4, 0.0)
    ids = torch.cat([text_ids, image_ids], 1)
    bare = sampling.denoise_joint(model, noise, text, ids, sigmas=torch.tensor(sig))
    out = sampling.denoise(model, noise, text, image_ids, text_ids, recipe=SamplingRecipe(sigmas=sig))
    assert torch.equal(out, bare)
    seen = []
    stepped = sampling.denoise(model, noise, text, image_ids, text_ids,
                               recipe=SamplingRecipe(sigmas=sig),
                               on_step=lambda i, cur, vel: seen.append(i))
    assert seen == [0, 1, 2]
    # the update as its own launch is the epilogue's update: same roundings, same bits
    assert torch.equal(stepped, bare), show("on_step vs fused", metrics(stepped, bare))
    expect = ref.denoise(w, noise, text, ids, torch.tensor(sig), v, negative=negative, guidance=3.0)
    outs = {}
    for mode in ("sequential", "batched"):
        recipe = SamplingRecipe(variant="base", guidance=3.0, cfg_mode=mode, sigmas=sig)
        outs[mode] = sampling.denoise(model, noise, text, image_ids, text_ids, recipe=recipe,
                                      negative=negative)
        m = metrics(outs[mode], expect)
        print(show(f"CFG {mode} vs oracle", m))
        assert m["cos"] >= 0.999 and m["rel_l2"] <= 3e-2, show(mode, m)
    m = metrics(outs["sequential"], outs["batched"])
    print(show("sequential vs batched CFG", m))
    assert m["rel_l2"] <= 1e-3, show("sequential vs batched", m)


def test_ltx_state_loop_matches_bare_loop(cuda_device):
    v = lcfg.BASELINE_VIDEO.with_blocks(2)
    w = ltx_weights(v, seed=41)
    grid = (2, 6, 8)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=42)
    context = normal((1, 32, v.context_dim), seed=43)
    pos = lref.pixel_coords(lref.patch_grid_bounds(*grid))
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[4:]
    model = LTXVideoTransformer(w, v, cuda_device)
    bare = ldn.denoise_video(model, latent, context, pos, sigmas)
    dev_latent = latent.to(cuda_device)
    state = ldn.LatentState(latent=dev_latent, denoise_mask=None, positions=pos)
    video, _ = ldn.denoise_loop(state, None, sigmas, transformer=model,
                                video_context=context.to(cuda_device))
    assert torch.equal(video.latent, bare)
    assert torch.equal(state.latent, dev_latent)
    m = metrics(video.latent - latent.to(cuda_device),
                lref.denoise(w, latent, context, pos, sigmas, v) - latent)
    assert m["cos"] >= 0.999, show("LTX state loop update vs oracle", m)


def test_linear_rows_residual_in_the_epilogue(cuda_device):
    """mpp_linear.linear_rows (kinomlx/kernels/mpp_linear.py:592-611): residual + the rounded
    product, the add done in the GEMM epilogue, equals the product rounded then added."""
    from kinomlx_b200.kernels import mpp_linear

    x = normal((3, 70, 256), seed=51).to(cuda_device)
    w = normal((384, 256), seed=52, std=0.05).to(cuda_device)
    b = normal((384,), seed=53).to(cuda_device)
    r = normal((3, 70, 384), seed=54).to(cuda_device)
    got = mpp_linear.linear_rows(x, w, b, residual=r)
    plain = mpp_linear.linear(x, w, b, transposed=True)
    assert torch.equal(got, (plain.float() + r.float()).to(torch.bfloat16))
    assert torch.equal(mpp_linear.linear_rows(x, w, b), plain)
