"""Each CUDA kernel against a plain PyTorch fp32 restatement of the same op on identical inputs.

Tolerances: the bf16 parity gate is a max relative error <= 2e-2 per op; attention follows the
reference's own test bar (relative L2 < 6e-3 against fp32 SDPA for bf16 inputs,
tests/models/ltx2/test_dense_attention.py:15 in the reference).
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def _randn(shape, seed, scale=1.0):
    return (torch.randn(shape, generator=_gen(seed)) * scale).to(BF)


def _max_rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    out = out.float().cpu()
    ref = ref.float().cpu()
    return float((out - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def _rel_l2(out: torch.Tensor, ref: torch.Tensor) -> float:
    out = out.float().cpu()
    ref = ref.float().cpu()
    return float((out - ref).norm() / ref.norm().clamp_min(1e-30))


# ------------------------------------------------------------------------------------ GEMM
@pytest.mark.parametrize(
    ("batch", "m", "n", "k"),
    [
        (1, 128, 256, 64),
        (1, 300, 264, 200),
        (1, 1024, 64, 3072),
        (2, 517, 384, 128),
        (1, 4608, 3072, 3072),
        (1, 1536, 12288, 3072),
    ],
)
def test_linear_matches_fp32(cuda_device, batch, m, n, k):
    from kinomlx_b200 import ops

    x = _randn((batch, m, k), 1)
    w = _randn((n, k), 2, 0.02)
    bias = _randn((n,), 3, 0.1)
    ref = (x.float() @ w.float().T + bias.float()).to(BF)
    out = ops.linear(x.to(cuda_device), w.to(cuda_device), bias=bias.to(cuda_device))
    torch.cuda.synchronize()
    assert _max_rel(out, ref) <= 2e-2
    # same fp32 sum, one rounding: almost every element is bit-identical
    same = (out.cpu() == ref).float().mean().item()
    assert same > 0.95


def test_linear_strided_views_and_epilogues(cuda_device):
    from kinomlx_b200 import ops

    dev = cuda_device
    batch, m, k, n = 2, 200, 256, 512
    big = _randn((batch, m, 3 * k), 4).to(dev)
    x = big[:, :, k : 2 * k]  # strided view, row stride 3k
    w = _randn((n, k), 5, 0.05).to(dev)
    bias = _randn((n,), 6, 0.1).to(dev)
    xf, wf, bf = x.float().cpu(), w.float().cpu(), bias.float().cpu()
    proj = (xf @ wf.T + bf).to(BF).float()

    # GELU from column 256 on
    out = ops.linear(x, w, bias=bias, kind=ops.EPI_GELU, act_col_begin=256)
    g = proj.clone()
    t = g[..., 256:]
    g[..., 256:] = 0.5 * t * (1 + torch.tanh((0.7978845608028654 * (t + 0.044715 * t**3)).clamp(-10, 10)))
    assert _max_rel(out, g.to(BF)) <= 2e-2

    # gated residual, in place
    resid = _randn((batch, m, n), 7).to(dev)
    gate = _randn((batch, n), 8).to(dev)
    expect = (resid.float().cpu() + (gate.float().cpu()[:, None, :] * proj).to(BF).float()).to(BF)
    ops.linear(x, w, resid, bias=bias, kind=ops.EPI_GATED_RESIDUAL, residual=resid, gate=gate)
    torch.cuda.synchronize()
    assert _max_rel(resid, expect) <= 2e-2

    # Euler epilogue
    sample = _randn((batch, m, n), 9).to(dev)
    dt = -0.25
    v = proj.to(BF)
    inc = (torch.tensor(dt).to(BF) * v).float()
    expect = (sample.float().cpu() + inc).to(BF)
    out = ops.linear(x, w, bias=bias, kind=ops.EPI_EULER, dt=dt, sample=sample)
    assert _max_rel(out, expect) <= 2e-2

    # 2 * sigmoid gate logits
    out = ops.linear(x, w, bias=bias, kind=ops.EPI_SIGMOID2)
    assert _max_rel(out, (2 * torch.sigmoid(proj)).to(BF)) <= 2e-2


def test_linear_refuses_unaligned_widths(cuda_device):
    from kinomlx_b200 import ops

    x = torch.zeros((4, 12), dtype=BF, device=cuda_device)
    w = torch.zeros((16, 12), dtype=BF, device=cuda_device)
    with pytest.raises(RuntimeError, match="KINO_ENOTSUPPORTED"):
        ops.linear(x, w)


# ------------------------------------------------------------------------------------ attention
def _sdpa_ref(q, k, v, heads):
    tq, tk = q.shape[-2], k.shape[-2]
    d = q.shape[-1] // heads
    b = q.shape[0]
    qh = q.float().cpu().reshape(b, tq, heads, d).transpose(1, 2)
    kh = k.float().cpu().reshape(b, tk, heads, d).transpose(1, 2)
    vh = v.float().cpu().reshape(b, tk, heads, d).transpose(1, 2)
    s = (qh @ kh.transpose(-1, -2)) * d**-0.5
    o = torch.softmax(s, dim=-1) @ vh
    return o.transpose(1, 2).reshape(b, tq, heads * d)


@pytest.mark.parametrize(
    ("tq", "tk"),
    [(7, 7), (16, 16), (33, 33), (517, 517), (300, 1024), (1, 300), (517, 33), (40, 5)],
)
def test_attention_ragged_matches_fp32_sdpa(cuda_device, tq, tk):
    from kinomlx_b200 import ops

    heads = 2
    q = _randn((1, tq, heads * 128), 11)
    k = _randn((1, tk, heads * 128), 12)
    v = _randn((1, tk, heads * 128), 13)
    out = torch.empty_like(q).to(cuda_device)
    ops.attention([q.to(cuda_device)], [k.to(cuda_device)], [v.to(cuda_device)], [out], heads=heads)
    torch.cuda.synchronize()
    assert _rel_l2(out, _sdpa_ref(q, k, v, heads)) < 6e-3


def test_attention_two_segments_equal_concatenation(cuda_device):
    from kinomlx_b200 import ops

    dev = cuda_device
    heads, nt, ni, batch = 3, 130, 257, 2
    qkv_t = _randn((batch, nt, 3 * heads * 128), 21, 2.0).to(dev)
    qkv_i = _randn((batch, ni, 3 * heads * 128), 22, 2.0).to(dev)
    w = heads * 128
    seg = lambda t, j: t[:, :, j * w : (j + 1) * w]
    out_t = torch.empty((batch, nt, w), dtype=BF, device=dev)
    out_i = torch.empty((batch, ni, w), dtype=BF, device=dev)
    ops.attention(
        [seg(qkv_t, 0), seg(qkv_i, 0)],
        [seg(qkv_t, 1), seg(qkv_i, 1)],
        [seg(qkv_t, 2), seg(qkv_i, 2)],
        [out_t, out_i],
        heads=heads,
    )
    q = torch.cat([seg(qkv_t, 0), seg(qkv_i, 0)], dim=1)
    k = torch.cat([seg(qkv_t, 1), seg(qkv_i, 1)], dim=1)
    v = torch.cat([seg(qkv_t, 2), seg(qkv_i, 2)], dim=1)
    ref = _sdpa_ref(q, k, v, heads)
    assert _rel_l2(torch.cat([out_t, out_i], dim=1), ref) < 6e-3


@pytest.mark.parametrize(
    ("batch", "tq", "tk", "heads"),
    [(1, 7, 7, 2), (2, 300, 517, 3), (1, 517, 33, 2), (1, 1, 300, 4), (1, 1024, 126, 32)],
)
def test_attention_head_dim_64_matches_fp32_sdpa(cuda_device, batch, tq, tk, heads):
    """64-wide heads (the reference's audio stream and its audio/video cross-attention, 32 x 64),
    ragged query and key counts, batch 2."""
    from kinomlx_b200 import ops

    q = _randn((batch, tq, heads * 64), 31)
    k = _randn((batch, tk, heads * 64), 32)
    v = _randn((batch, tk, heads * 64), 33)
    out = torch.empty_like(q).to(cuda_device)
    ops.attention([q.to(cuda_device)], [k.to(cuda_device)], [v.to(cuda_device)], [out], heads=heads)
    torch.cuda.synchronize()
    assert _rel_l2(out, _sdpa_ref(q, k, v, heads)) < 6e-3


def test_dense_attention_surface_head_dim_64(cuda_device):
    """The reference dense-attention contract with dim 64: q (Tq, H*64), k and v (Tk, H*64)
    (kinomlx/models/ltx2/kernels/dense_attention.py:87-151), two key segments equal to one."""
    from kinomlx_b200 import ops
    from kinomlx_b200.kernels import dense_attention

    heads, tq, tk = 32, 300, 126
    q, k, v = _randn((tq, heads * 64), 34), _randn((tk, heads * 64), 35), _randn((tk, heads * 64), 36)
    dev = cuda_device
    assert dense_attention.applies(q[None].to(dev), k[None].to(dev), heads=heads)
    out = dense_attention.dense_attention(q.to(dev), k.to(dev), v.to(dev), heads=heads)
    ref = _sdpa_ref(q[None], k[None], v[None], heads)[0]
    assert _rel_l2(out, ref) < 6e-3
    split = torch.empty((1, tq, heads * 64), dtype=BF, device=dev)
    ops.attention([q[None].to(dev)], [k[None, :50].to(dev), k[None, 50:].to(dev)],
                  [v[None, :50].to(dev), v[None, 50:].to(dev)], [split], heads=heads)
    assert _rel_l2(split[0], ref) < 6e-3


def test_attention_full_size_flux(cuda_device):
    from kinomlx_b200 import ops

    heads, n = 24, 4608
    q = _randn((1, n, heads * 128), 31).to(cuda_device)
    k = _randn((1, n, heads * 128), 32).to(cuda_device)
    v = _randn((1, n, heads * 128), 33).to(cuda_device)
    out = torch.empty_like(q)
    ops.attention([q], [k], [v], [out], heads=heads)
    # compare 2 heads on the CPU
    ref = _sdpa_ref(q[..., :256], k[..., :256], v[..., :256], 2)
    assert _rel_l2(out[..., :256], ref) < 6e-3


# ------------------------------------------------------------------------------------ norms
def test_adaln_layer_and_rms(cuda_device):
    from kinomlx_b200 import ops

    dev = cuda_device
    batch, rows, dim = 2, 37, 3072
    x = _randn((batch, rows, dim), 41, 3.0)
    shift = _randn((batch, dim), 42)
    scale = _randn((batch, dim), 43)
    xf = x.float()
    ln = ((xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, unbiased=False, keepdim=True) + 1e-6)).to(BF)
    expect = ((ln * (1 + scale[:, None, :])) + shift[:, None, :])  # bf16 ops
    out = ops.adaln(x.to(dev), shift.to(dev), scale.to(dev), norm=ops.NORM_LAYER)
    assert _max_rel(out, expect) <= 2e-2
    rms = (xf / torch.sqrt((xf * xf).mean(-1, keepdim=True) + 1e-6)).to(BF)
    expect = (rms * (1 + scale[:, None, :])) + shift[:, None, :]
    out = ops.adaln(x.to(dev), shift.to(dev), scale.to(dev), norm=ops.NORM_RMS)
    assert _max_rel(out, expect) <= 2e-2


def test_rms_norm_weighted(cuda_device):
    from kinomlx_b200 import ops

    x = _randn((2, 5, 256), 20260816, 2.0)
    w = _randn((256,), 51)
    xf = x.float()
    ref = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6) * (w.float() + 1.0)).to(BF)
    out = ops.rms_norm(x.to(cuda_device), w.to(cuda_device), 1e-6, weight_offset=1.0)
    assert _max_rel(out, ref) <= 2e-2


def test_qk_norm_rope_per_head_pairs(cuda_device):
    from kinomlx_b200 import ops

    heads, tokens = 3, 50
    x = _randn((1, tokens, heads * 128), 61, 2.0)
    w = _randn((128,), 62)
    ang = torch.randn((tokens, 64), generator=_gen(63))
    ang = ang.repeat_interleave(2, dim=-1)
    cos, sin = torch.cos(ang), torch.sin(ang)
    xf = x.float().reshape(1, tokens, heads, 128)
    n = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6) * w.float()).to(BF).float()
    pairs = n.reshape(1, tokens, heads, 64, 2)
    perp = torch.stack([-pairs[..., 1], pairs[..., 0]], -1).reshape(n.shape)
    ref = (n * cos[None, :, None] + perp * sin[None, :, None]).to(BF).reshape(1, tokens, -1)
    xd = x.to(cuda_device)
    ops.qk_norm_rope(
        xd, heads=heads, weight=w.to(cuda_device), norm=ops.QKNORM_PER_HEAD, rope=ops.ROPE_PAIRS,
        cos=cos.to(cuda_device), sin=sin.to(cuda_device),
    )
    assert _max_rel(xd, ref) <= 2e-2


def test_qk_norm_rope_full_row_split(cuda_device):
    from kinomlx_b200 import ops

    heads, tokens = 4, 33
    x = _randn((2, tokens, heads * 128), 71, 2.0)
    w = _randn((heads * 128,), 72)
    ang = torch.randn((1, heads, tokens, 64), generator=_gen(73))
    cos, sin = torch.cos(ang), torch.sin(ang)
    xf = x.float()
    n = (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-6) * w.float()).to(BF).float()
    nh = n.reshape(2, tokens, heads, 128).transpose(1, 2)
    a, c = nh[..., :64], nh[..., 64:]
    out = torch.cat([a * cos - c * sin, a * sin + c * cos], -1)
    ref = out.transpose(1, 2).reshape(2, tokens, heads * 128).to(BF)
    xd = x.to(cuda_device)
    ops.qk_norm_rope(
        xd, heads=heads, weight=w.to(cuda_device), norm=ops.QKNORM_FULL_ROW, rope=ops.ROPE_SPLIT,
        cos=cos.to(cuda_device), sin=sin.to(cuda_device),
    )
    assert _max_rel(xd, ref) <= 2e-2


def test_split_rope_bit_exact_self_test_recipe(cuda_device):
    """The reference kernel's own self-test inputs (kinomlx/kernels/split_rope.py:120-136)."""
    from kinomlx_b200 import ops

    batch, heads, tokens, half = 2, 3, 7, 5
    count = batch * tokens * heads * 2 * half
    value = (torch.sin(torch.arange(count, dtype=torch.float32) * 0.7310585) * 3.0).to(BF)
    value = value.reshape(batch, tokens, heads * 2 * half)
    angles = torch.arange(tokens * heads * half, dtype=torch.float32) * 0.4142135
    angles = angles.reshape(1, tokens, heads, half).transpose(1, 2)
    cos, sin = torch.cos(angles), torch.sin(angles)
    hf = value.reshape(batch, tokens, heads, 2 * half).transpose(1, 2).float()
    first, second = hf[..., :half], hf[..., half:]
    graph = torch.cat([first * cos - second * sin, first * sin + second * cos], -1)
    graph = graph.transpose(1, 2).reshape(value.shape).to(BF)
    out = ops.split_rope(value.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device))
    assert torch.equal(out.cpu(), graph)


@pytest.mark.parametrize("batch,heads,tokens,half,table_batch",
                         [(1, 32, 300, 64, 1), (2, 3, 17, 8, 2), (2, 2, 5, 12, 1)])
def test_split_rope_vector_path_bit_exact(cuda_device, batch, heads, tokens, half, table_batch):
    """half % 4 == 0 runs the four-pair kernel: bit-identical to the reference graph
    (kinomlx/kernels/split_rope.py:87-98), with shared and per-batch tables."""
    from kinomlx_b200 import ops

    value = _randn((batch, tokens, heads * 2 * half), 51)
    angles = torch.rand((table_batch, heads, tokens, half),
                        generator=torch.Generator().manual_seed(52)) * 6.0
    cos, sin = torch.cos(angles), torch.sin(angles)
    hf = value.reshape(batch, tokens, heads, 2 * half).transpose(1, 2).float()
    first, second = hf[..., :half], hf[..., half:]
    graph = torch.cat([first * cos - second * sin, first * sin + second * cos], -1)
    graph = graph.transpose(1, 2).reshape(value.shape).to(BF)
    out = ops.split_rope(value.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device))
    assert torch.equal(out.cpu(), graph)


@pytest.mark.parametrize("channels", [64, 128, 512, 1024, 96])
def test_pixel_norm_widths(cuda_device, channels):
    """Every PixelNorm (+ SiLU) form: the vector kernels (64..1024, powers of two) and the
    warp-per-voxel kernel (other widths), against the stepwise bf16 oracle
    (kinomlx/kernels/fused_ops.py:460-476, blocks.py:165-168)."""
    from kinomlx_b200 import ops
    from oracle import fused_ops as fo

    x = _randn((3, 7, 11, channels), 53)
    for silu in (False, True):
        exp = fo.pixel_norm(x, dim=-1, eps=1e-8)
        if silu:
            exp = fo.silu(exp)
        out = ops.pixel_norm(x.to(cuda_device), 1e-8, silu=silu).cpu()
        assert _max_rel(out, exp) <= 2e-2
        assert (out == exp).float().mean() > 0.97


# ------------------------------------------------------------------------------------ elementwise
def test_gelu_silu_bounds(cuda_device):
    """On the reference's grid (tests/kernels/test_fused_ops.py: linspace(-8, 8, 65536) in bf16).
    GELU: the device evaluates 0.5 (1 + tanh u) as the logistic 1 / (1 + e^(-2u)), which is
    exact where the fp32 tanh formula cancels (the negative tail), so it is held to the float64
    GELU (bf16 equal almost everywhere) and to the per-op bound against the fp32 formula (max
    relative error <= 2e-2; one bf16 ulp elementwise). SiLU: equal to the fp32 formula, the
    reference's bound (max abs 0 in bf16)."""
    from kinomlx_b200 import ops

    x = torch.linspace(-8, 8, 65536).to(BF)
    xf, x64 = x.float(), x.double()
    gelu32 = (0.5 * xf * (1 + torch.tanh((0.7978845608028654 * (xf + 0.044715 * xf**3)).clamp(-10, 10)))).to(BF)
    gelu64 = (x64 * torch.special.expit(2 * 0.7978845608028654 * (x64 + 0.044715 * x64**3))).to(BF)
    silu = (xf / (1 + torch.exp(-xf))).to(BF)
    g = ops.gelu_tanh(x.to(cuda_device)).cpu()
    s = ops.silu(x.to(cuda_device)).cpu()
    assert (g == gelu64).float().mean() > 0.99
    assert (g.float() - gelu32.float()).abs().max() <= 2e-2 * gelu32.float().abs().max()
    # where the fp32 formula underflows to -0 the exact value is below 1e-6 in magnitude
    assert ((g.float() - gelu32.float()).abs() <= gelu32.float().abs() * 2.0**-7 + 1e-6).all()
    assert torch.equal(s, silu)


def test_cfg_and_euler_rounding_order(cuda_device):
    from kinomlx_b200 import ops

    cond = _randn((4096, 64), 81)
    uncond = _randn((4096, 64), 82)
    ref = uncond + 4.0 * (cond - uncond)  # bf16 ops
    out = ops.cfg_combine(cond.to(cuda_device), uncond.to(cuda_device), 4.0)
    assert torch.equal(out.cpu(), ref)
    # Klein Euler (kinomlx/models/flux2/sampling.py:109-113)
    x = _randn((4096, 64), 83)
    v = _randn((4096, 64), 84)
    dt = float(torch.tensor(0.75, dtype=torch.float32) - torch.tensor(1.0, dtype=torch.float32))
    inc = torch.tensor(dt, dtype=torch.float32).to(BF) * v
    ref = (x.float() + inc.float()).to(BF)
    out = ops.euler_velocity(x.to(cuda_device), v.to(cuda_device), dt)
    assert torch.equal(out.cpu(), ref)
    # LTX X0 + Euler
    sigma, nxt = 0.909375, 0.725
    x0 = (x.float() - sigma * v.float()).to(BF)
    ratio = torch.tensor(nxt / sigma, dtype=torch.float32)
    ref = (x0.float() + ratio * (x.float() - x0.float())).to(BF)
    out = ops.euler_x0(x.to(cuda_device), v.to(cuda_device), sigma, nxt)
    assert torch.equal(out.cpu(), ref)


def test_gemv_and_timestep_embedding(cuda_device):
    from kinomlx_b200 import ops

    t = torch.tensor([500.0, 999.0], dtype=torch.float32)
    freq = torch.exp(-math.log(10000) * torch.arange(128, dtype=torch.float32) / 128)
    ang = t[:, None] * freq
    ref = torch.cat([torch.cos(ang), torch.sin(ang)], -1).to(BF)
    emb = ops.timestep_embedding(t.to(cuda_device), 256)
    assert _max_rel(emb, ref) <= 2e-2
    x = _randn((2, 3072), 91)
    w = _randn((18432, 3072), 92, 0.02)
    b = _randn((18432,), 93, 0.1)
    xs = (x.float() / (1 + torch.exp(-x.float()))).to(BF)
    ref = ((xs.float() @ w.float().T).to(BF).float() + b.float()).to(BF)
    out = ops.gemv(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), silu_input=True)
    assert _max_rel(out, ref) <= 2e-2


def test_linear_fused_qk_norm_rope_and_gelu(cuda_device):
    """[k | v | q | mlp] projection with per-head RMSNorm + pair RoPE on k and q and GELU on the
    MLP columns in one epilogue, against the separate fp32 formulas."""
    from kinomlx_b200 import ops

    dev = cuda_device
    m, k, heads = 300, 256, 2
    d = heads * 128
    n = 3 * d + 512
    x = _randn((1, m, k), 101)
    w = _randn((n, k), 102, 0.05)
    nq = _randn((128,), 103) + 1
    nk = _randn((128,), 104) + 1
    ang = torch.randn((m + 40, 64), generator=_gen(105)).repeat_interleave(2, dim=-1)
    cos, sin = torch.cos(ang), torch.sin(ang)
    proj = (x.float() @ w.float().T).to(BF).float()[0]

    def norm_rope(part, weight, off):
        h = part.reshape(m, heads, 128)
        y = (h * torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-6) * weight.float()).to(BF).float()
        c, s = cos[off : off + m, None], sin[off : off + m, None]
        pairs = y.reshape(m, heads, 64, 2)
        perp = torch.stack([-pairs[..., 1], pairs[..., 0]], -1).reshape(y.shape)
        return (y * c + perp * s).reshape(m, d)

    t = proj[:, 3 * d :]
    gelu = 0.5 * t * (1 + torch.tanh((0.7978845608028654 * (t + 0.044715 * t**3)).clamp(-10, 10)))
    expect = torch.cat([norm_rope(proj[:, :d], nk, 40), proj[:, d : 2 * d],
                        norm_rope(proj[:, 2 * d : 3 * d], nq, 40), gelu], dim=1).to(BF)
    out = ops.linear(x.to(dev), w.to(dev), kind=ops.EPI_GELU, act_col_begin=3 * d,
                     qk_norm=[(0, nk.to(dev)), (2 * d, nq.to(dev))], norm_width=d,
                     rope=(ops.RopeTables(cos.to(dev), sin.to(dev)), 40))
    assert _max_rel(out[0], expect) <= 2e-2
    assert (out[0].cpu() == expect).float().mean() > 0.95


@pytest.mark.parametrize("batch,m,n,k", [(1, 768, 512, 256), (1, 2560, 2048, 512), (2, 768, 768, 256)])
def test_linear_lead_rows_use_their_own_weight_norm_and_gate(cuda_device, batch, m, n, k):
    """One launch over a joint [text | image] sequence: the first 256 rows of every batch entry
    take the lead weight and gate, the rest the main ones; equal to two separate products."""
    from kinomlx_b200 import ops

    dev = cuda_device
    lead = 256
    x = _randn((batch, m, k), 201)
    w, wl = _randn((n, k), 202, 0.05), _randn((n, k), 203, 0.05)
    gate, gate_l = _randn((batch, n), 204), _randn((batch, n), 205)
    res = _randn((batch, m, n), 206)
    expect = torch.empty((batch, m, n), dtype=torch.float32)
    for b in range(batch):
        for rows, wt, g in ((slice(0, lead), wl, gate_l), (slice(lead, m), w, gate)):
            y = (x[b, rows].float() @ wt.float().T).to(BF).float()
            expect[b, rows] = res[b, rows].float() + (g[b].float() * y).to(BF).float()
    out = res.clone().to(dev)
    ops.linear(x.to(dev), w.to(dev), out, kind=ops.EPI_GATED_RESIDUAL, residual=out,
               gate=gate.to(dev), lead_w=wl.to(dev), lead_rows=lead, lead_gate=gate_l.to(dev))
    assert _max_rel(out, expect.to(BF)) <= 2e-2
    assert (out.cpu() == expect.to(BF)).float().mean() > 0.95
