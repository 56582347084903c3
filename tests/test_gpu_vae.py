"""Device video-VAE kernels and decoder against the CPU oracle on identical seeded inputs.

Conv parity: fp32 accumulation rounded once to bf16 on both sides, so nearly every element is
bit-identical; the gate is max relative error <= 2e-2. Decoder parity: cosine >= 0.999 and
relative L2 <= 2e-2 on the fp32 video. Miniature decoders keep the CPU oracle in seconds.
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle import fused_ops as fo
from oracle import video_vae as ref
from kinomlx_b200 import ops
from kinomlx_b200.ltx2 import video_vae as vae
from kinomlx_b200.synthetic import make_weights, normal

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _metrics(out, expect):
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return (float((o - e).norm() / e.norm()), float((o - e).abs().max() / e.abs().max()),
            float(torch.nn.functional.cosine_similarity(o, e, dim=0)))


@pytest.mark.parametrize(
    ("f", "h", "w", "cin", "n", "causal", "stride", "residual"),
    [
        (5, 9, 11, 64, 64, False, (1, 1, 1), False),
        (5, 9, 11, 64, 64, True, (1, 1, 1), True),
        (2, 8, 8, 128, 128, False, (1, 1, 1), False),
        (3, 16, 16, 128, 48, True, (1, 1, 1), False),
        (4, 6, 10, 128, 256, True, (2, 2, 2), False),
        (3, 20, 36, 64, 128, False, (1, 2, 2), False),
        (3, 12, 8, 64, 64, False, (2, 1, 1), False),
        # enough voxel boxes for a wave of CTA pairs: M = 256 tiles over two SMs, each SM loading
        # its own box and half of the weight rows (an odd box count leaves the odd CTA of the
        # last pair on zero fill; 96 and 320 outputs leave part of a half-block past the end)
        (8, 64, 128, 64, 128, True, (1, 1, 1), True),
        (11, 36, 80, 128, 64, False, (1, 1, 1), False),
        (9, 40, 72, 64, 256, True, (1, 1, 1), True),
        (7, 44, 76, 128, 96, False, (1, 1, 1), False),
        (6, 40, 64, 64, 320, True, (1, 1, 1), False),
        (8, 64, 64, 128, 48, True, (1, 1, 1), False),  # the decoder's conv_out width, in pairs
        # 128-channel pairs on rows of >= 128 voxels: one input row per (kt, kh) serving the
        # three kw taps (a full row, and a row of 200 with a partial second box)
        (5, 24, 200, 128, 128, False, (1, 1, 1), True),
        (6, 32, 128, 128, 128, True, (1, 1, 1), False),
        (4, 40, 128, 128, 256, True, (1, 1, 1), True),  # the same for 256 channels
        (3, 32, 128, 256, 512, True, (1, 2, 2), False),  # and under depth-to-space
    ],
)
def test_conv3d_matches_oracle(cuda_device, f, h, w, cin, n, causal, stride, residual):
    x = normal((1, f, h, w, cin), seed=1)
    wt = normal((n, 3, 3, 3, cin), seed=2, std=0.05)
    b = normal((n,), seed=3, std=0.1)
    sub = math.prod(stride)
    if sub == 1:
        exp = ref.conv3d(x, wt, b, causal)
        res = normal(exp.shape, seed=4) if residual else None
        if res is not None:
            exp = exp + res
        out = ops.conv3d(x.to(cuda_device).contiguous(), wt.to(cuda_device), b.to(cuda_device),
                         causal=causal, residual=None if res is None else res[0].to(cuda_device))
    else:
        cout = n // sub
        p = {"u.conv.weight": wt, "u.conv.bias": b}
        exp = ref.upsample(p, "u", x, stride, cin // cout, ref.VaeVariant(causal=causal))
        wd = wt.reshape(cout, sub, 3, 3, 3, cin).transpose(0, 1).reshape(wt.shape)
        bd = b.reshape(cout, sub).transpose(0, 1).reshape(-1)
        out = ops.conv3d(x.to(cuda_device).contiguous(), wd.to(cuda_device).contiguous(),
                         bd.to(cuda_device).contiguous(), causal=causal, stride=stride)
    torch.cuda.synchronize()
    exp = exp[0]
    assert tuple(out.shape) == tuple(exp.shape)
    rel_l2, max_rel, cos = _metrics(out, exp)
    assert max_rel <= 2e-2, (rel_l2, max_rel)
    assert (out.cpu() == exp).float().mean() > 0.95


@pytest.mark.parametrize(
    ("f", "h", "w", "cin", "n", "causal", "stride", "residual"),
    [
        # output tiles filling under half of the SMs with a long reduction: split-K over CTAs
        (4, 8, 8, 256, 512, True, (1, 1, 1), True),
        (3, 6, 8, 1024, 256, False, (1, 1, 1), False),
        (3, 8, 8, 512, 1024, True, (1, 2, 2), False),
        (5, 8, 8, 512, 128, True, (1, 1, 1), True),
        (3, 6, 8, 256, 96, False, (1, 1, 1), False),
    ],
)
def test_conv3d_split_k_matches_oracle(cuda_device, f, h, w, cin, n, causal, stride, residual):
    """Split-K convs (fp32 partial sums added in split order by the CTA that completes the tile)
    against the oracle, against the same conv without a workspace, and a second launch on the
    same workspace (its tile counters back at zero) giving identical bytes."""
    dev = cuda_device
    x = normal((1, f, h, w, cin), seed=41)
    wt = normal((n, 3, 3, 3, cin), seed=42, std=0.05)
    b = normal((n,), seed=43, std=0.1)
    sub = math.prod(stride)
    ws = ops.conv_workspace(dev)
    if sub == 1:
        exp = ref.conv3d(x, wt, b, causal)
        res = normal(exp.shape, seed=44) if residual else None
        if res is not None:
            exp = exp + res
        args = (x.to(dev).contiguous(), wt.to(dev), b.to(dev))
        kw = dict(causal=causal, residual=None if res is None else res[0].to(dev))
    else:
        cout = n // sub
        p = {"u.conv.weight": wt, "u.conv.bias": b}
        exp = ref.upsample(p, "u", x, stride, cin // cout, ref.VaeVariant(causal=causal))
        wd = wt.reshape(cout, sub, 3, 3, 3, cin).transpose(0, 1).reshape(wt.shape)
        bd = b.reshape(cout, sub).transpose(0, 1).reshape(-1)
        args = (x.to(dev).contiguous(), wd.to(dev).contiguous(), bd.to(dev).contiguous())
        kw = dict(causal=causal, stride=stride)
    split = ops.conv3d(*args, workspace=ws, **kw)
    again = ops.conv3d(*args, workspace=ws, **kw)
    whole = ops.conv3d(*args, **kw)
    torch.cuda.synchronize()
    assert int(ws[:16384].view(torch.int32).abs().sum()) == 0  # counters reset
    assert torch.equal(split, again)
    exp = exp[0]
    rel_l2, max_rel, _ = _metrics(split, exp)
    assert max_rel <= 2e-2, (rel_l2, max_rel)
    assert (split.cpu() == exp).float().mean() > 0.95
    assert (split == whole).float().mean() > 0.95


def test_pixel_and_group_norm_silu(cuda_device):
    x = normal((3, 7, 9, 256), seed=5, std=2.0)
    exp = fo.silu(fo.pixel_norm(x, dim=-1, eps=1e-8))
    out = ops.pixel_norm(x.to(cuda_device), 1e-8, silu=True)
    assert _metrics(out, exp)[1] <= 2e-2
    assert (out.cpu() == exp).float().mean() > 0.97
    wt = normal((256,), seed=6, std=0.5) + 1
    bs = normal((256,), seed=7, std=0.1)
    x1 = x.reshape(1, 21, 9, 256)  # one video: statistics over every voxel of the batch item
    exp = fo.silu(fo.group_norm(x1, 32, wt.to(BF), bs, 1e-6))
    out = ops.group_norm(x1.to(cuda_device), 32, wt.to(BF).to(cuda_device), bs.to(cuda_device), 1e-6, silu=True)
    assert _metrics(out, exp)[1] <= 2e-2
    # the statistics reduce in a fixed order: a second call gives the same bits
    again = ops.group_norm(x1.to(cuda_device), 32, wt.to(BF).to(cuda_device), bs.to(cuda_device), 1e-6, silu=True)
    assert torch.equal(out, again)
    x128 = normal((1, 66, 17, 128), seed=8)
    exp = fo.group_norm(x128, 32, torch.ones(128, dtype=BF), torch.zeros(128, dtype=BF), 1e-6)
    out = ops.group_norm(x128.to(cuda_device), 32, torch.ones(128, dtype=BF, device=cuda_device),
                         torch.zeros(128, dtype=BF, device=cuda_device), 1e-6)
    assert _metrics(out, exp)[1] <= 2e-2


MINI = (("res", 1), ("d2s", (2, 2, 2), 2), ("res", 1), ("d2s", (1, 2, 2), 1), ("res", 1))


@pytest.mark.parametrize("norm,causal", [("pixel", False), ("group32", True)])
def test_mini_decoder_matches_oracle(cuda_device, norm, causal):
    v = vae.VaeVariant(norm=norm, causal=causal, top_width=256, blocks=MINI)
    rv = ref.VaeVariant(norm=norm, causal=causal, top_width=256, blocks=MINI)
    w = make_weights(vae.vae_weight_specs(v), seed=11)
    latent = normal((1, 128, 3, 4, 6), seed=12)
    exp = ref.decode(w, latent, rv)
    dec = vae.VideoDecoder(w, v, cuda_device)
    out = dec.decode(latent.to(cuda_device), tile=None)
    assert tuple(out.shape) == tuple(exp.shape)
    rel_l2, max_rel, cos = _metrics(out, exp)
    assert cos >= 0.999 and rel_l2 <= 2e-2, (rel_l2, max_rel, cos)


def test_mini_tiled_decode_matches_oracle(cuda_device):
    v = vae.VaeVariant(norm="group32", causal=True, top_width=256, blocks=MINI)
    rv = ref.VaeVariant(norm="group32", causal=True, top_width=256, blocks=MINI)
    w = make_weights(vae.vae_weight_specs(v), seed=13)
    latent = normal((1, 128, 2, 7, 10), seed=14)
    exp = ref.decode_tiled(w, latent, rv, tile=4, overlap=1, scale=16)
    dec = vae.VideoDecoder(w, v, cuda_device)
    out = dec.decode(latent.to(cuda_device), tile=4, overlap=1)
    rel_l2, max_rel, cos = _metrics(out, exp)
    assert cos >= 0.999 and rel_l2 <= 2e-2, (rel_l2, max_rel, cos)


def test_config5_shapes_first_stages_run(cuda_device):
    """Full-width LTX-2.3 decoder on one config-5 tile (8 x 8 latents, 16 frames), weights
    drawn on the GPU: output shape (1, 3, 121, 256, 256), finite."""
    v = vae.BASELINE_VAE
    w = make_weights(vae.vae_weight_specs(v), seed=0, device=cuda_device)
    dec = vae.VideoDecoder(w, v, cuda_device)
    latent = normal((1, 128, 16, 8, 8), seed=1, device=cuda_device)
    out = dec.decode(latent, tile=None)
    torch.cuda.synchronize()
    assert tuple(out.shape) == (1, 3, 121, 256, 256)
    assert bool(torch.isfinite(out).all())


@pytest.mark.parametrize(
    ("f", "h", "w", "cin", "n", "causal", "stride", "residual"),
    [
        (5, 9, 11, 64, 128, True, (1, 1, 1), True),
        (4, 6, 10, 128, 256, True, (2, 2, 2), False),
        (3, 20, 36, 64, 1024, False, (1, 1, 1), False),
        (2, 16, 40, 128, 64, True, (1, 1, 1), False),
        (11, 36, 80, 64, 128, True, (1, 1, 1), True),
        (4, 8, 8, 512, 512, True, (1, 1, 1), True),  # split-K: statistics from the last split
        (3, 8, 8, 256, 512, True, (1, 2, 2), False),
    ],
)
def test_group_norm_from_conv_statistics(cuda_device, f, h, w, cin, n, causal, stride, residual):
    """GroupNorm(32) + SiLU from the statistics the conv's epilogue gathered (Chan-merged count,
    mean and m2 per group) against the two-pass fp32 GroupNorm of the same conv output (oracle
    formula): the same bf16 values almost everywhere, per-op bound max relative error 2e-2."""
    dev = cuda_device
    x = normal((f, h, w, cin), seed=31, device=dev)
    wt = normal((n, 3, 3, 3, cin), seed=32, device=dev, std=0.05)
    bias = normal((n,), seed=33, device=dev)
    sub = math.prod(stride)
    co = n // sub
    res = normal((f, h, w, co), seed=34, device=dev) if residual else None
    stats = ops.conv_stats_buffer(dev)
    y = ops.conv3d(x, wt, bias, causal=causal, stride=stride, residual=res, stats=stats,
                   workspace=ops.conv_workspace(dev))
    gw = normal((co,), seed=35, device=dev) + 1
    gb = normal((co,), seed=36, device=dev)
    got = ops.group_norm_from_stats(y, gw, gb, 1e-6, stats, silu=True)
    expect = fo.group_norm(y.reshape(1, -1, co).cpu(), 32, gw.cpu(), gb.cpu(), 1e-6)
    expect = fo.silu(expect).reshape(y.shape)
    _, max_rel, cosine = _metrics(got, expect)
    assert max_rel <= 2e-2 and cosine >= 0.9999, (max_rel, cosine)
    assert (got.cpu() == expect).float().mean() > 0.97
