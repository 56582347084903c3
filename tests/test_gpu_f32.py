"""fp32 parity mode against the CPU oracle in fp32 (BASELINE: per-op max relative error <= 1e-4
in fp32 mode; config 1 asks for the double block in fp32 as well as bf16).

Max relative error here is max |device - oracle| / max |oracle| over the whole output, the same
measure the bf16 tests use. Every case compares the fp32 CUDA kernels (through the C ABI) with the
oracle's fp32 restatement on identical seeded inputs drawn on the CPU.
"""

from __future__ import annotations

import pytest
import torch

from oracle import flux2 as ref
from oracle import fused_ops as rops
from oracle import ltx2 as lref
from oracle import video_vae as vref
from kinomlx_b200 import _lib
from kinomlx_b200 import ops_f32 as f
from kinomlx_b200.flux2 import config as fcfg
from kinomlx_b200.flux2 import sampling
from kinomlx_b200.flux2.transformer import rotary_positions
from kinomlx_b200.flux2.transformer_f32 import Flux2TransformerF32
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2 import denoise as ldn
from kinomlx_b200.ltx2.transformer import precompute_freqs_cis
from kinomlx_b200.ltx2 import video_vae as vae
from kinomlx_b200.ltx2.transformer_f32 import LTXVideoTransformerF32
from kinomlx_b200.ltx2.video_vae_f32 import VideoDecoderF32
from kinomlx_b200.synthetic import flux_weights, ltx_weights, make_weights, normal

pytestmark = pytest.mark.gpu
F32 = torch.float32
TOL = 1e-4  # BASELINE's fp32-mode gate


def _max_rel(out: torch.Tensor, expect: torch.Tensor) -> float:
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return float((o - e).abs().max() / e.abs().max())


def _cos(out: torch.Tensor, expect: torch.Tensor) -> float:
    o, e = out.float().cpu().flatten(), expect.float().cpu().flatten()
    return float(torch.nn.functional.cosine_similarity(o.double(), e.double(), dim=0))


def _r(shape, seed, std=1.0):
    return normal(shape, seed=seed, dtype=F32, std=std)


@pytest.mark.parametrize("m,n,k,batch", [(77, 200, 36, 1), (300, 384, 1024, 2), (1, 18432, 3072, 1)])
def test_linear_f32_plain_and_bias(cuda_device, m, n, k, batch):
    x, w, b = _r((batch, m, k), 1), _r((n, k), 2, 0.02), _r((n,), 3)
    out = f.linear(x.to(cuda_device), w.to(cuda_device), bias=b.to(cuda_device))
    assert _max_rel(out, rops.linear(x, w, b)) <= TOL


def test_linear_f32_epilogues(cuda_device):
    """GELU on a column range, gated residual with a per-batch gate (in place), Euler update."""
    dev = cuda_device
    batch, m, n, k = 2, 133, 264, 520
    x, w = _r((batch, m, k), 4), _r((n, k), 5, 0.02)
    y = rops.linear(x, w)
    out = f.linear(x.to(dev), w.to(dev), kind=_lib.EPI_GELU, act_col_begin=128)
    expect = torch.cat([y[..., :128], rops.gelu_approx(y[..., 128:])], -1)
    assert _max_rel(out, expect) <= TOL
    res, gate = _r((batch, m, n), 6), _r((batch, n), 7)
    res_d = res.to(dev)
    f.linear(x.to(dev), w.to(dev), res_d, kind=_lib.EPI_GATED_RESIDUAL, residual=res_d,
             gate=gate.to(dev))
    assert _max_rel(res_d, res + gate[:, None] * y) <= TOL
    cur = _r((batch, m, n), 8)
    cur_d = cur.to(dev)
    f.linear(x.to(dev), w.to(dev), cur_d, kind=_lib.EPI_EULER, dt=-0.25, sample=cur_d)
    assert _max_rel(cur_d, ref.euler_step(cur, y, torch.tensor(-0.25))) <= TOL


@pytest.mark.parametrize("batch,tq,tk,heads", [(2, 77, 130, 2), (1, 1536, 1536, 24)])
def test_attention_f32_matches_sdpa(cuda_device, batch, tq, tk, heads):
    q, k, v = _r((batch, tq, heads * 128), 9), _r((batch, tk, heads * 128), 10), _r((batch, tk, heads * 128), 11)
    sh = lambda t: t.reshape(*t.shape[:2], heads, 128).transpose(1, 2)
    expect = rops.sdpa(sh(q), sh(k), sh(v), scale=128**-0.5).transpose(1, 2).reshape(q.shape)
    qd = q.to(cuda_device)
    out = f.attention(qd, k.to(cuda_device), v.to(cuda_device), qd, heads=heads)  # over q
    assert _max_rel(out, expect) <= TOL


@pytest.mark.parametrize("dim", [200, 3072])
@pytest.mark.parametrize("norm", [_lib.NORM_LAYER, _lib.NORM_RMS, _lib.NORM_NONE])
def test_adaln_f32(cuda_device, dim, norm):
    batch, rows = 2, 37
    x, shift, scale = _r((batch, rows, dim), 12), _r((batch, 1, dim), 13), _r((batch, 1, dim), 14)
    if norm == _lib.NORM_LAYER:
        base = rops.layer_norm(x, 1e-6)
    elif norm == _lib.NORM_RMS:
        base = rops.rms_norm(x, None, 1e-6)
    else:
        base = x
    expect = base * (1 + scale) + shift
    out = f.adaln(x.to(cuda_device), shift[:, 0].to(cuda_device), scale[:, 0].to(cuda_device),
                  norm=norm)
    assert _max_rel(out, expect) <= TOL


def test_qk_norm_rope_f32(cuda_device):
    """Per-head RMSNorm with weight, then the adjacent-pair rotation, on a column slice of a wider
    row and at a table offset (the image rows of a joint sequence)."""
    heads, tokens, offset = 3, 50, 7
    v = fcfg.BASELINE
    ids = torch.cat([torch.zeros((1, offset, 2), dtype=torch.int64), ref.image_ids(5, 10, 2)], 1)
    cos4, sin4 = ref.rotary_positions(ids, v)
    cos, sin = rotary_positions(ids, v)
    x = _r((2, tokens, 3 * heads * 128), 15)
    weight = 1 + _r((128,), 16, 0.1)
    sl = x[..., heads * 128 : 2 * heads * 128].reshape(2, tokens, heads, 128)
    expect = ref.rotate(rops.rms_norm(sl, weight, 1e-6), cos4[:, offset:], sin4[:, offset:])
    xd = x.to(cuda_device)
    f.qk_norm_rope(xd[..., heads * 128 : 2 * heads * 128], heads=heads, weight=weight.to(cuda_device),
                   norm=_lib.QKNORM_PER_HEAD, rope=_lib.ROPE_PAIRS, cos=cos.to(cuda_device),
                   sin=sin.to(cuda_device), table_offset=offset)
    got = xd.cpu()
    assert _max_rel(got[..., heads * 128 : 2 * heads * 128], expect.reshape(2, tokens, -1)) <= TOL
    assert torch.equal(got[..., : heads * 128], x[..., : heads * 128])  # untouched neighbours
    assert torch.equal(got[..., 2 * heads * 128 :], x[..., 2 * heads * 128 :])


def test_elementwise_f32(cuda_device):
    dev = cuda_device
    x, y = _r((4099,), 17, 3.0), _r((4099,), 18)
    assert _max_rel(f.gelu_tanh(x.to(dev)), rops.gelu_approx(x)) <= TOL
    assert _max_rel(f.silu(x.to(dev)), rops.silu(x)) <= TOL
    assert _max_rel(f.cfg_combine(x.to(dev), y.to(dev), 4.0), y + 4.0 * (x - y)) <= TOL
    assert _max_rel(f.euler_velocity(x.to(dev), y.to(dev), -0.125),
                    ref.euler_step(x, y, torch.tensor(-0.125))) <= TOL
    h = _r((2, 9, 2 * 96), 19)
    hd = h.to(dev)
    out = f.swiglu(hd, out=hd[..., :96])  # in place over the gate half
    assert _max_rel(out, ref.swiglu(h)) <= TOL
    t = torch.tensor([500.0, 875.0])
    got = f.timestep_embedding(t.to(dev), 256)
    freq = torch.exp(-torch.log(torch.tensor(10000.0)) * torch.arange(128, dtype=F32) / 128)
    ang = t[:, None] * freq
    assert _max_rel(got, torch.cat([torch.cos(ang), torch.sin(ang)], -1)) <= TOL


def _block_inputs(v, seed, nt, h, wd):
    w = flux_weights(v, seed=seed, dtype=F32)
    ids = torch.cat([torch.zeros((1, nt, 2), dtype=torch.int64), ref.image_ids(h, wd, 2)], 1)
    return w, ids


def test_config1_double_block_f32(cuda_device):
    """BASELINE config 1 in fp32: one MMDiT double block, 512 text + 1024 image tokens, hidden
    3072, 24 heads, t = 0.5, seed 0, weights N(0, 0.02) drawn in fp32."""
    v = fcfg.BASELINE.with_blocks(1, 0)
    w, ids = _block_inputs(v, 0, 512, 32, 32)
    image = _r((1, 1024, v.dim), 1)
    text = _r((1, 512, v.dim), 2)
    t = torch.tensor([0.5], dtype=F32)
    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    im = ref.modulation(w, "double_stream_modulation_img", emb)
    tm = ref.modulation(w, "double_stream_modulation_txt", emb)
    exp_img, exp_txt = ref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)

    dev = cuda_device
    model = Flux2TransformerF32(w, v, dev)
    cos, sin = rotary_positions(ids, v)
    img, txt = model.double_block(0, image.to(dev), text.to(dev), (t * 1000).to(dev),
                                  cos.to(dev), sin.to(dev))
    for out, exp in ((img, exp_img), (txt, exp_txt)):
        assert out.dtype == F32
        assert _max_rel(out, exp) <= TOL, _max_rel(out, exp)
        assert _cos(out, exp) >= 0.99999


@pytest.mark.parametrize("mlp", ["gelu_tanh", "swiglu"])
def test_single_block_f32(cuda_device, mlp):
    if mlp == "gelu_tanh":
        v = fcfg.BASELINE.with_blocks(0, 1)
    else:
        v = fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072, rope_axes=(64, 64),
                             rope_theta=10000.0, in_channels=64, context_dim=512,
                             double_blocks=0, single_blocks=1)
    nt, h, wd = 100, 12, 20
    w, ids = _block_inputs(v, 5, nt, h, wd)
    value = _r((1, nt + h * wd, v.dim), 6)
    t = torch.tensor([0.75], dtype=F32)
    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    sm = ref.modulation(w, "single_stream_modulation", emb)
    expect = ref.single_block(w, 0, value, sm, cos4, sin4, v)
    dev = cuda_device
    model = Flux2TransformerF32(w, v, dev)
    cos, sin = rotary_positions(ids, v)
    out = model.single_block(0, value.to(dev), nt, (t * 1000).to(dev), cos.to(dev), sin.to(dev))
    assert _max_rel(out, expect) <= TOL, _max_rel(out, expect)


def test_klein_double_block_f32(cuda_device):
    """SwiGLU (gate first) double block at hidden 1024 / 8 heads, batch 2 (per-entry modulation)."""
    v = fcfg.FluxVariant(dim=1024, heads=8, mlp="swiglu", mlp_hidden=3072, rope_axes=(64, 64),
                         rope_theta=10000.0, in_channels=64, context_dim=512, double_blocks=1,
                         single_blocks=0)
    nt, h, wd = 48, 8, 10
    w, ids = _block_inputs(v, 30, nt, h, wd)
    image, text = _r((2, h * wd, v.dim), 31), _r((2, nt, v.dim), 32)
    t = torch.tensor([0.25, 0.875], dtype=F32)
    cos4, sin4 = ref.rotary_positions(ids, v)
    emb = ref.timestep_embedding(w, t * 1000)
    im = ref.modulation(w, "double_stream_modulation_img", emb)
    tm = ref.modulation(w, "double_stream_modulation_txt", emb)
    exp_img, exp_txt = ref.double_block(w, 0, image, text, im, tm, cos4, sin4, v)
    dev = cuda_device
    model = Flux2TransformerF32(w, v, dev)
    cos, sin = rotary_positions(ids, v)
    img, txt = model.double_block(0, image.to(dev), text.to(dev), (t * 1000).to(dev),
                                  cos.to(dev), sin.to(dev))
    assert _max_rel(img, exp_img) <= TOL and _max_rel(txt, exp_txt) <= TOL


@pytest.mark.parametrize("cfg", [False, True])
def test_denoise_f32_matches_oracle(cuda_device, cfg):
    """The whole fp32 trajectory (1 double + 1 single block at hidden 512, 3 Euler steps, with and
    without batched CFG): final latent within the per-op bound and cosine >= 0.999 (BASELINE)."""
    v = fcfg.FluxVariant(dim=512, heads=4, mlp="gelu_tanh", mlp_hidden=2048, rope_axes=(64, 64),
                         rope_theta=10000.0, in_channels=64, context_dim=256, double_blocks=1,
                         single_blocks=1)
    nt, h, wd = 32, 8, 8
    w, ids = _block_inputs(v, 40, nt, h, wd)
    noise = _r((1, h * wd, v.in_channels), 41)
    text = _r((1, nt, v.context_dim), 42)
    negative = _r((1, nt, v.context_dim), 43) if cfg else None
    sigmas = ref.linear_sigmas(3)
    guidance = 4.0 if cfg else 1.0
    expect = ref.denoise(w, noise, text, ids, sigmas, v, negative=negative, guidance=guidance)
    model = Flux2TransformerF32(w, v, cuda_device)
    out = sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.linear_sigmas(3),
                           negative=negative, guidance=guidance)
    assert out.dtype == F32
    assert _max_rel(out, expect) <= TOL, _max_rel(out, expect)
    assert _cos(out, expect) >= 0.999


def test_linear_f32_ltx_epilogues(cuda_device):
    """2 * sigmoid (the LTX head gates) and X0 + Euler (the LTX sampler update)."""
    dev = cuda_device
    batch, m, n, k = 2, 70, 136, 264
    x, w, b = _r((batch, m, k), 60), _r((n, k), 61, 0.05), _r((n,), 62)
    y = rops.linear(x, w, b)
    got = f.linear(x.to(dev), w.to(dev), bias=b.to(dev), kind=_lib.EPI_SIGMOID2)
    assert _max_rel(got, 2.0 * torch.sigmoid(y)) <= TOL
    cur = _r((batch, m, n), 63)
    sigma, nxt = lref.DISTILLED_STAGE_1_SIGMAS[6], lref.DISTILLED_STAGE_1_SIGMAS[7]
    expect = lref.euler_step(cur, lref.to_denoised(cur, sigma, y), sigma, nxt)
    cur_d = cur.to(dev)
    ratio = float(torch.tensor(nxt / sigma, dtype=F32))
    f.linear(x.to(dev), w.to(dev), cur_d, bias=b.to(dev), kind=_lib.EPI_EULER_X0,
             sigma=float(torch.tensor(sigma, dtype=F32)), ratio=ratio, sample=cur_d)
    assert _max_rel(cur_d, expect) <= TOL


@pytest.mark.parametrize("rope", [True, False])
def test_qk_norm_rope_f32_full_row_split(cuda_device, rope):
    """RMSNorm over the whole 4096-wide row with its weight, then the split-half rotation per
    head (the LTX q/k path), on a column slice of a wider row; without RoPE, the cross-attention
    q/k norm."""
    v = lcfg.BASELINE_VIDEO
    pos = lref.pixel_coords(lref.patch_grid_bounds(2, 3, 5))
    cos, sin = precompute_freqs_cis(pos, v)
    tokens, d = cos.shape[2], v.dim
    x = _r((1, tokens, 3 * d), 64)
    wt = 1 + _r((d,), 65, 0.1)
    expect = rops.rms_norm(x[..., d : 2 * d], wt, v.eps)
    if rope:
        expect = lref.apply_split_rotary_emb(expect, cos, sin)
    xd = x.to(cuda_device)
    f.qk_norm_rope(xd[..., d : 2 * d], heads=v.heads, weight=wt.to(cuda_device),
                   norm=_lib.QKNORM_FULL_ROW, rope=_lib.ROPE_SPLIT if rope else _lib.ROPE_NONE,
                   cos=cos.to(cuda_device) if rope else None,
                   sin=sin.to(cuda_device) if rope else None, eps=v.eps)
    got = xd.cpu()
    assert _max_rel(got[..., d : 2 * d], expect) <= TOL
    assert torch.equal(got[..., :d], x[..., :d]) and torch.equal(got[..., 2 * d :], x[..., 2 * d :])


def test_attention_f32_gate_and_add_rows(cuda_device):
    """The per-head output gate of the LTX attention (cross-attention shape: 90 queries, 33
    context keys) and the modulation-table add."""
    dev = cuda_device
    batch, tq, tk, heads = 2, 90, 33, 3
    q, k, v = _r((batch, tq, heads * 128), 66), _r((batch, tk, heads * 128), 67), _r((batch, tk, heads * 128), 68)
    gate = 2.0 * torch.sigmoid(_r((batch, tq, heads), 69))
    sh = lambda t: t.reshape(*t.shape[:2], heads, 128).transpose(1, 2)
    att = rops.sdpa(sh(q), sh(k), sh(v), scale=128**-0.5).transpose(1, 2)
    expect = (att * gate[..., None]).reshape(q.shape)
    out = f.attention(q.to(dev), k.to(dev), v.to(dev), heads=heads, gate=gate.to(dev))
    assert _max_rel(out, expect) <= TOL
    table, row = _r((9, 520), 70), _r((520,), 71)
    assert torch.equal(f.add_rows(table.to(dev), row.to(dev)).cpu(), table + row)


def _ltx_positions(f_, h, w):
    return lref.pixel_coords(lref.patch_grid_bounds(f_, h, w))


def test_ltx_block_velocity_f32(cuda_device):
    """One full-width LTX-2 video block (hidden 4096, 32 heads: the q/k norm spans 4096
    channels) with gated self- and cross-attention, in fp32: velocity within 1e-4 of the oracle."""
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=80, dtype=F32)
    grid = (2, 4, 6)
    latent = _r((1, grid[0] * grid[1] * grid[2], v.in_channels), 81)
    context = _r((1, 40, v.context_dim), 82)
    pos = _ltx_positions(*grid)
    sigma = lref.DISTILLED_STAGE_1_SIGMAS[5]
    expect = lref.forward(w, latent, context, sigma, pos, v, dtype=F32)
    model = LTXVideoTransformerF32(w, v, cuda_device)
    out = model.run(model.prepare(context, pos), latent.to(cuda_device), sigma).clone()
    assert out.dtype == F32
    assert _max_rel(out, expect) <= TOL, _max_rel(out, expect)
    assert _cos(out, expect) >= 0.99999


def test_ltx_denoise_f32(cuda_device):
    """Two blocks at hidden 1024 / 8 heads over the last three distilled stage-1 steps with
    X0 + Euler in the final projection, fp32 end to end, batch 2."""
    v = lcfg.LTXVariant(dim=1024, heads=8, context_dim=1024, blocks=2)
    w = ltx_weights(v, seed=83, dtype=F32)
    grid = (2, 4, 4)
    latent = _r((2, grid[0] * grid[1] * grid[2], v.in_channels), 84)
    context = _r((2, 24, v.context_dim), 85)
    pos = _ltx_positions(*grid)
    sigmas = lref.DISTILLED_STAGE_1_SIGMAS[5:]
    expect = lref.denoise(w, latent, context, pos, sigmas, v)
    model = LTXVideoTransformerF32(w, v, cuda_device)
    out = ldn.denoise_video(model, latent, context, pos, sigmas)
    assert out.dtype == F32
    assert _max_rel(out, expect) <= TOL, _max_rel(out, expect)
    assert _cos(out, expect) >= 0.999


@pytest.mark.parametrize(
    ("f_", "h", "w", "cin", "n", "causal", "stride", "residual"),
    [
        (5, 9, 11, 64, 64, False, (1, 1, 1), False),
        (5, 9, 11, 64, 64, True, (1, 1, 1), True),
        (2, 5, 7, 16, 40, True, (1, 1, 1), True),
        (3, 16, 16, 128, 48, True, (1, 1, 1), False),
        (4, 6, 10, 128, 256, True, (2, 2, 2), False),
        (3, 20, 36, 64, 128, False, (1, 2, 2), False),
        (3, 12, 8, 64, 64, False, (2, 1, 1), False),
    ],
)
def test_conv3d_f32(cuda_device, f_, h, w, cin, n, causal, stride, residual):
    """3x3x3 conv with the reference's temporal replicate / spatial zero padding, bias, residual
    and depth-to-space upsampling, fp32 (kinomlx/models/ltx2/video_vae/blocks.py:97-139,
    decoder.py:80-121)."""
    dev = cuda_device
    x = _r((1, f_, h, w, cin), 90)
    wt = _r((n, 3, 3, 3, cin), 91, 0.05)
    b = _r((n,), 92, 0.1)
    sub = stride[0] * stride[1] * stride[2]
    if sub == 1:
        exp = vref.conv3d(x, wt, b, causal)
        res = _r(exp.shape, 93) if residual else None
        if res is not None:
            exp = exp + res
        out = f.conv3d(x.to(dev), wt.to(dev), b.to(dev), causal=causal,
                       residual=None if res is None else res[0].to(dev))
    else:
        cout = n // sub
        exp = vref.upsample({"u.conv.weight": wt, "u.conv.bias": b}, "u", x, stride, cin // cout,
                            vref.VaeVariant(causal=causal))
        wd = wt.reshape(cout, sub, 3, 3, 3, cin).transpose(0, 1).reshape(wt.shape).contiguous()
        bd = b.reshape(cout, sub).transpose(0, 1).reshape(-1).contiguous()
        out = f.conv3d(x.to(dev), wd.to(dev), bd.to(dev), causal=causal, stride=stride)
    exp = exp[0]
    assert tuple(out.shape) == tuple(exp.shape)
    assert _max_rel(out, exp) <= TOL, _max_rel(out, exp)


@pytest.mark.parametrize("channels", [128, 96, 256])
def test_vae_norms_f32(cuda_device, channels):
    """Stepwise PixelNorm + SiLU and affine GroupNorm(32) + SiLU in fp32
    (kinomlx/kernels/fused_ops.py:375-409, 460-476)."""
    dev = cuda_device
    x = _r((1, 5, 7, 9, channels), 94, 2.0)
    exp = rops.silu(rops.pixel_norm(x, dim=-1, eps=1e-8))
    assert _max_rel(f.pixel_norm(x.to(dev), 1e-8, silu=True), exp) <= TOL
    if channels % 32 == 0:
        wt, bs = 1 + _r((channels,), 95, 0.3), _r((channels,), 96, 0.1)
        x1 = x.reshape(1, 5, 63, channels)
        exp = rops.silu(rops.group_norm(x1, 32, wt, bs, 1e-6))
        got = f.group_norm(x1.to(dev), 32, wt.to(dev), bs.to(dev), 1e-6, silu=True)
        assert _max_rel(got, exp) <= TOL


VAE_MINI = (("res", 1), ("d2s", (2, 2, 2), 2), ("res", 1), ("d2s", (1, 2, 2), 1), ("res", 1))


@pytest.mark.parametrize("norm,causal", [("pixel", False), ("group32", True)])
def test_vae_decoder_f32(cuda_device, norm, causal):
    """A miniature decoder (top width 256, both depth-to-space kinds, residual blocks) in fp32,
    the whole video within 1e-4 of the oracle's fp32 decode."""
    v = vae.VaeVariant(norm=norm, causal=causal, top_width=256, blocks=VAE_MINI)
    rv = vref.VaeVariant(norm=norm, causal=causal, top_width=256, blocks=VAE_MINI)
    w = make_weights(vae.vae_weight_specs(v), seed=97, dtype=F32)
    latent = _r((1, 128, 3, 4, 6), 98)
    exp = vref.decode(w, latent, rv, dtype=F32)
    out = VideoDecoderF32(w, v, cuda_device).decode(latent.to(cuda_device), tile=None)
    assert tuple(out.shape) == tuple(exp.shape)
    assert _max_rel(out, exp) <= TOL, _max_rel(out, exp)


def test_vae_tiled_decode_f32(cuda_device):
    """The spatial tiler with trapezoid blending in fp32 (tiling.py:1053-1386)."""
    v = vae.VaeVariant(norm="group32", causal=True, top_width=256, blocks=VAE_MINI)
    rv = vref.VaeVariant(norm="group32", causal=True, top_width=256, blocks=VAE_MINI)
    w = make_weights(vae.vae_weight_specs(v), seed=99, dtype=F32)
    latent = _r((1, 128, 2, 7, 10), 100)
    exp = vref.decode_tiled(w, latent, rv, tile=4, overlap=1, scale=16, dtype=F32)
    out = VideoDecoderF32(w, v, cuda_device).decode(latent.to(cuda_device), tile=4, overlap=1)
    assert _max_rel(out, exp) <= TOL, _max_rel(out, exp)


def test_f32_refusals(cuda_device):
    """Contract violations come back as errors, not silent work: a k that is not a multiple of 4,
    a misaligned row stride, an epilogue with no fp32 form, a table too short for the rows."""
    dev = cuda_device
    with pytest.raises(RuntimeError, match="ENOTSUPPORTED"):
        f.linear(torch.zeros((4, 6), device=dev), torch.zeros((8, 6), device=dev))
    with pytest.raises(ValueError, match="no fp32 form"):
        f.linear(torch.zeros((4, 8), device=dev), torch.zeros((8, 8), device=dev),
                 kind=_lib.EPI_SWIGLU)
    x = torch.zeros((1, 5, 128), device=dev)
    tab = torch.zeros((1, 4, 128), device=dev)
    with pytest.raises(RuntimeError, match="EINVAL"):
        f.qk_norm_rope(x, heads=1, weight=None, norm=_lib.QKNORM_NONE, rope=_lib.ROPE_PAIRS,
                       cos=tab, sin=tab)
