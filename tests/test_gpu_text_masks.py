"""Padded text masks on the B200: the attention kernels' additive key bias and the LTX-2 classes'
cross-attention under a mask, against torch fp32 and the CPU oracle
(kinomlx/models/ltx2/transformer/preprocessing.py:85-96, attention.py:164-186).

A padded key's bias (-3.39e38) sends its probability to exactly 0 in the kernel, so a mask that
pads the tail of the context must give the same bits as the context cut to its tokens (the same
key blocks, the same maxima, zeros added to the sums): that is asserted with torch.equal. A row
whose keys are all masked averages them uniformly, as the finite bias does in the reference.
Gates against the oracle are the block tests' (relative L2 1e-2 / 3e-2, cosine 0.999)."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import ltx2 as lref
from kinomlx_b200 import ops, ops_f32
from kinomlx_b200.ltx2 import av_transformer as avm
from kinomlx_b200.ltx2.config import LTXVariant
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer, context_key_bias
from kinomlx_b200.synthetic import ltx_av_weight_specs, ltx_weights, make_weights, normal
from parity_metrics import metrics, show

pytestmark = pytest.mark.gpu
MIN = -3.3895313892515355e38


def _masked_reference(q, k, v, heads, bias):
    """torch fp32: softmax(q k^T / sqrt(d) + bias) v, per head."""
    b, tq, width = q.shape
    d = width // heads
    sh = lambda t: t.float().reshape(t.shape[0], t.shape[1], heads, d).transpose(1, 2)
    s = sh(q) @ sh(k).transpose(-1, -2) / math.sqrt(d) + bias[:, None, None, : k.shape[1]]
    return (torch.softmax(s, -1) @ sh(v)).transpose(1, 2).reshape(b, tq, width)


@pytest.mark.parametrize("head_dim", [128, 64])
def test_attention_key_bias(cuda_device, head_dim):
    heads, tq, tk = 2, 300, 200  # a partial last key block
    gen = torch.Generator().manual_seed(head_dim)
    q, k, v = (torch.randn((3, n, heads * head_dim), generator=gen).to(torch.bfloat16)
               for n in (tq, tk, tk))
    mask = torch.ones((3, tk), dtype=torch.int32)
    mask[0, torch.randperm(tk, generator=gen)[:70]] = 0  # holes anywhere
    mask[1] = 0  # every key masked: a uniform average
    bias = context_key_bias(mask, 3, tk, "cpu")
    bias[2, :tk] = torch.rand((tk,), generator=gen) * -6.0  # a float bias on the third prompt
    out = torch.empty_like(q).to(cuda_device)
    ops.attention([q.to(cuda_device)], [k.to(cuda_device)], [v.to(cuda_device)], [out],
                  heads=heads, key_bias=bias.to(cuda_device))
    torch.cuda.synchronize()
    expect = _masked_reference(q, k, v, heads, bias)
    uniform = v[1].float().mean(0)  # every key masked: the reference itself averages them
    assert float((expect[1] - uniform).abs().max()) < 1e-5
    for b in range(3):
        m = metrics(out[b], expect[b])
        assert m["rel_l2"] <= 1e-2 and m["max_norm"] <= 2e-2, show(f"prompt {b}", m)


def test_fp32_attention_key_bias(cuda_device):
    heads, tq, tk = 2, 130, 77
    gen = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn((2, n, heads * 128), generator=gen) for n in (tq, tk, tk))
    bias = context_key_bias(torch.tensor([[1] * 50 + [0] * 27, [0] * 77]), 2, tk, "cpu",
                            dtype=torch.float32)
    got = ops_f32.attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), heads=heads,
                            key_bias=bias.to(cuda_device))
    expect = _masked_reference(q, k, v, heads, bias)
    err = float((got.cpu() - expect).abs().max() / expect.abs().max())
    assert err <= 1e-4, err


def _ltx_case(cuda_device, seed):
    v = LTXVariant(dim=1024, heads=8, context_dim=1024, blocks=2)
    w = ltx_weights(v, seed=seed)
    grid = (2, 4, 8)
    latent = normal((2, grid[0] * grid[1] * grid[2], v.in_channels), seed=seed + 1)
    context = normal((2, 40, v.context_dim), seed=seed + 2)
    pos = lref.pixel_coords(lref.patch_grid_bounds(*grid))
    return v, w, latent, context, pos, LTXVideoTransformer(w, v, cuda_device)


def test_ltx_padded_prompt_equals_cut_prompt(cuda_device):
    """Both prompts padded after 25 tokens: the masked forward is the forward on the first 25
    context tokens, bit for bit; and it matches the oracle's masked forward."""
    v, w, latent, context, pos, model = _ltx_case(cuda_device, 300)
    mask = torch.zeros((2, 40), dtype=torch.int64)
    mask[:, :25] = 1
    sigma = lref.DISTILLED_STAGE_1_SIGMAS[5]
    dl = latent.to(cuda_device)
    masked = model.run(model.prepare(context, pos, context_mask=mask), dl, sigma).clone()
    cut = model.run(model.prepare(context[:, :25], pos), dl, sigma).clone()
    assert torch.equal(masked, cut)
    plain = model.run(model.prepare(context, pos), dl, sigma).clone()
    assert not torch.equal(masked, plain)
    expect = lref.forward(w, latent, context, sigma, pos, v, context_mask=mask)
    m = metrics(masked, expect)
    assert m["rel_l2"] <= 1e-2 and m["cos"] >= 0.999, show("masked forward vs oracle", m)


def test_ltx_loop_with_uneven_padding_matches_oracle(cuda_device):
    """Prompts padded after 31 and 12 tokens (different per batch item, one launch), through the
    reference's denoise_loop over the last three distilled steps."""
    from kinomlx_b200.ltx2 import denoise as ldn

    v, w, latent, context, pos, model = _ltx_case(cuda_device, 310)
    mask = torch.zeros((2, 40), dtype=torch.bool)
    mask[0, :31] = True
    mask[1, :12] = True
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    state = ldn.LatentState(latent=latent.to(cuda_device), denoise_mask=None, positions=pos)
    video, _ = ldn.denoise_loop(state, None, sigmas, transformer=model,
                                video_context=context.to(cuda_device), video_context_mask=mask)
    expect = lref.denoise(w, latent, context, pos, sigmas, v, context_mask=mask)
    m = metrics(video.latent - latent.to(cuda_device), expect - latent)
    assert m["rel_l2"] <= 3e-2 and m["cos"] >= 0.999, show("masked loop update vs oracle", m)


def test_av_padded_prompts_equal_cut_prompts(cuda_device):
    """The joint audio/video block: each stream's text mask, against the same streams with the
    contexts cut to their tokens (bit for bit)."""
    video = LTXVariant(dim=1024, heads=8, context_dim=1024, blocks=1)
    audio = LTXVariant(dim=512, heads=8, head_dim=64, context_dim=512, max_pos=(20,), blocks=1)
    w = make_weights(ltx_av_weight_specs(video, audio, 1), seed=320)
    vlat = normal((1, 2 * 4 * 4, video.in_channels), seed=321).to(cuda_device)
    alat = normal((1, 20, audio.in_channels), seed=322).to(cuda_device)
    vctx, actx = normal((1, 24, video.dim), seed=323), normal((1, 18, audio.dim), seed=324)
    vpos = lref.pixel_coords(lref.patch_grid_bounds(2, 4, 4))
    start = torch.arange(20, dtype=torch.float32) * 0.04
    apos = torch.stack([start, start + 0.04], -1)[None, None]
    vmask = torch.tensor([[1] * 17 + [0] * 7])
    amask = torch.tensor([[1] * 9 + [0] * 9])
    model = avm.LTXAVTransformer(w, video, audio, cuda_device)
    sigma = lref.DISTILLED_STAGE_1_SIGMAS[5]
    prep = model.prepare(vctx, actx, vpos, apos, video_context_mask=vmask, audio_context_mask=amask)
    mv, ma = (t.clone() for t in model.run(prep, vlat, alat, sigma))
    cv, ca = (t.clone() for t in model.run(model.prepare(vctx[:, :17], actx[:, :9], vpos, apos),
                                           vlat, alat, sigma))
    assert torch.equal(mv, cv) and torch.equal(ma, ca)
