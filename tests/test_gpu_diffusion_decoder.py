"""LTX-2.5 diffusion video decoder on the B200 against the CPU oracle
(kinomlx/models/ltx2/video_vae/diffusion_decoder.py): the q/k/v preparation kernel against an
fp32 restatement, the strided copy against torch, the context stages and the whole decode
(padding to the minimum grid, trailing and ghost frames, crop) against oracle.diffusion_decoder,
a two-step x0 schedule, and batch entries decoded independently.

Gates: the q/k preparation within fp16 rounding of fp32 math (2e-3 of the largest value);
copies bit-exact; the decode's video within relative L2 3e-2 and cosine 0.999 of the oracle
(bf16 activations through eight blocks; the attention operands fp16)."""

from __future__ import annotations

import pytest
import torch

from oracle import diffusion_decoder as dref
from kinomlx_b200 import ops
from kinomlx_b200.ltx2.diffusion_decoder import (DiffusionDecoderConfig, DiffusionVideoDecoder,
                                                 patchify_spatial, rope_tables, unpatchify_spatial)
from kinomlx_b200.synthetic import diffusion_decoder_weights, normal
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu

CFG = DiffusionDecoderConfig(
    head_dim=64, stage_channels=(256, 128, 128, 64, 64), stage_depths=(1, 1, 1, 1, 2),
    stage_kernels=((3, 3, 3), (3, 3, 3), (3, 5, 5), (3, 5, 5)),
    upsample_strides=((1, 2, 2), (2, 1, 1), (2, 2, 2), (2, 2, 2)),
    upsample_channel_reductions=(2, 1, 2, 1), stage5_kernel=(3, 5, 5), patch_size=4,
    t_emb_dim=128, spatial_compression_ratio=32, temporal_compression_ratio=8,
    latent_channels=128)


@pytest.fixture(scope="module")
def model_and_weights(cuda_device):
    w = diffusion_decoder_weights(CFG, seed=11)
    return DiffusionVideoDecoder(w, CFG, cuda_device), w


def test_na_qkv_prepare_matches_fp32(cuda_device):
    grid, heads = (3, 5, 7), 2
    tokens = 3 * 5 * 7
    width = heads * 64
    qkv = normal((tokens, 3 * width + 64), seed=1)[:, : 3 * width + 64]
    wq = (1.0 + 0.1 * normal((64,), seed=2, dtype=torch.float32)).to(torch.bfloat16)
    wk = (1.0 + 0.1 * normal((64,), seed=3, dtype=torch.float32)).to(torch.bfloat16)
    tables = rope_tables(64, grid)
    q, k, v = ops.na_qkv_prepare(qkv.to(cuda_device), wq.to(cuda_device), wk.to(cuda_device),
                                 tables.to(cuda_device), grid, batch=1, heads=heads,
                                 section_pairs=(8, 12, 12), q_scale=0.125)
    torch.cuda.synchronize()

    def expect(cols, weight, scale):
        x = qkv[:, cols].float().reshape(1, *grid, heads, 64)
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * weight.float() * scale
        return dref.rope3d(x, 64)

    eq = expect(slice(0, width), wq, 0.125)
    ek = expect(slice(width, 2 * width), wk, 1.0)
    for got, exp, name in ((q, eq, "q"), (k, ek, "k")):
        err = float((got.float().cpu() - exp).abs().max() / exp.abs().max())
        assert err <= 2e-3, (name, err)
    assert torch.equal(v.cpu(), qkv[:, 2 * width : 3 * width].to(torch.float16).reshape(v.shape))


def test_copy_view_matches_torch(cuda_device):
    x = normal((3, 4, 5, 6, 7, 2), seed=5).to(cuda_device)
    perm = x.permute(3, 0, 5, 1, 4, 2)
    out = torch.empty(perm.shape, device=cuda_device, dtype=torch.bfloat16)
    ops.copy_view(perm, out)
    assert torch.equal(out, perm.contiguous())
    h = normal((1000, 64), seed=6, dtype=torch.float16).to(cuda_device)
    hb = torch.empty((1000, 64), device=cuda_device, dtype=torch.bfloat16)
    ops.copy_view(h, hb)
    assert torch.equal(hb, h.to(torch.bfloat16))
    f = normal((77, 33), seed=7, dtype=torch.float32).to(cuda_device)
    fb = torch.empty((77, 33), device=cuda_device, dtype=torch.bfloat16)
    ops.copy_view(f, fb)
    assert torch.equal(fb, f.to(torch.bfloat16))
    row = x[1:2, :, 2:3]  # broadcast along two axes, into a strided destination
    big = torch.zeros((3, 4, 4, 6, 7, 2), device=cuda_device, dtype=torch.bfloat16)
    ops.copy_view(row.expand(3, 4, 3, 6, 7, 2), big[:, :, 1:])
    assert torch.equal(big[:, :, 1:], row.expand(3, 4, 3, 6, 7, 2))
    assert not big[:, :, 0].any()


def test_neighborhood_attention_bf16_output(cuda_device):
    """The decoder's form of the attention: the same fp32 result rounded to bf16 once."""
    shape = (1, 5, 9, 17, 2, 64)
    q, k, v = (normal(shape, seed=s, dtype=torch.float16).to(cuda_device) for s in (51, 52, 53))
    q = q * 0.125
    half = ops.neighborhood_attention(q, k, v, window=(3, 5, 5))
    bf = torch.empty(shape, device=cuda_device, dtype=torch.bfloat16)
    ops.neighborhood_attention(q, k, v, window=(3, 5, 5), out=bf)
    torch.cuda.synchronize()
    diff = (bf.float() - half.float()).abs()
    assert float((diff / half.float().abs().clamp_min(1e-3)).max()) <= 2 ** -8


def test_patchify_matches_oracle(cuda_device):
    x = normal((2, 3, 5, 16, 24), seed=8)
    packed = patchify_spatial(x.to(cuda_device), 4)
    assert torch.equal(packed.cpu(), dref.patchify_spatial(x, 4))
    assert torch.equal(unpatchify_spatial(packed, 4).cpu(), x)


def test_context_stages_match_oracle(model_and_weights):
    model, w = model_and_weights
    latent = normal((1, 128, 2, 2, 3), seed=21, dtype=torch.float32)
    ctx, grid, _ = model.context(latent[0].to(model.device))
    torch.cuda.synchronize()
    padded, _ = dref.edge_pad_axis(latent, 2, 3, True)
    padded, _ = dref.edge_pad_axis(padded, 3, 3, False)
    padded, _ = dref.edge_pad_axis(padded, 4, 3, False)
    std = w["per_channel_statistics.std_of_means"].reshape(1, -1, 1, 1, 1)
    mean = w["per_channel_statistics.mean_of_means"].reshape(1, -1, 1, 1, 1)
    den = (padded.to(torch.bfloat16).float() * std + mean).to(torch.bfloat16)
    expect = dref.stage_4(dref.stages_1_to_3(den, w, CFG), w, CFG)
    assert tuple(expect.shape[1:4]) == grid
    m = metrics(ctx.reshape(expect.shape), expect)
    assert m["rel_l2"] <= 3e-2 and m["cos"] >= 0.999, show("context", m)


@pytest.mark.parametrize("latent_shape, steps", [((1, 128, 2, 2, 3), None), ((1, 128, 3, 3, 4), 2)])
def test_decode_matches_oracle(model_and_weights, latent_shape, steps):
    model, w = model_and_weights
    latent = normal(latent_shape, seed=31, dtype=torch.float32).to(torch.bfloat16)
    noise = normal(CFG.working_pixel_shape(latent_shape), seed=32)
    got = model(latent.to(model.device), noise.to(model.device), steps=steps)
    torch.cuda.synchronize()
    ops.device_status()
    expect = dref.decode(latent, noise, w, CFG, steps)
    assert tuple(got.shape) == tuple(expect.shape)
    m = metrics(got, expect)
    assert m["rel_l2"] <= 3e-2 and m["cos"] >= 0.999, show(f"decode {latent_shape}", m)


def test_batch_entries_decode_independently(model_and_weights):
    model, _ = model_and_weights
    shape = (2, 128, 2, 1, 2)
    latent = normal(shape, seed=41).to(model.device)
    noise = normal(CFG.working_pixel_shape(shape), seed=42).to(model.device)
    both = model(latent, noise)
    one = model(latent[1:], noise[1:])
    torch.cuda.synchronize()
    assert torch.equal(both[1:], one)
    assert not torch.equal(both[0], both[1])
