"""Device dequantisation of packed weights and packed LTX block linears against the oracle.

Dequantisation is exact in fp32 for the float modes and one fma for affine, rounded once, so the
device weight must equal the oracle's bit for bit. The quantised matmul and the packed LTX block
then follow the bf16 GEMM's own bounds (max relative error <= 2e-2, cosine >= 0.999).
"""

from __future__ import annotations

import pytest
import torch

from oracle import ltx2 as ref
from oracle import quantized as oq
from kinomlx_b200 import ops
from kinomlx_b200.ltx2 import config as lcfg
from kinomlx_b200.ltx2.transformer import LTXVideoTransformer
from kinomlx_b200.synthetic import ltx_weights, normal

pytestmark = pytest.mark.gpu


def _packed(mode, rows, cols, seed, std=0.05):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn((rows, cols), generator=g) * std
    gs, bits = oq.DEFAULTS[mode]
    words, scales, biases = oq.quantize(w, mode=mode, group_size=gs, bits=bits)
    return words, scales, biases, gs, bits


@pytest.mark.parametrize("mode", ["affine", "mxfp8", "mxfp4", "nvfp4"])
@pytest.mark.parametrize(("rows", "cols"), [(64, 128), (96, 320), (48, 32), (128, 4096)])
@pytest.mark.parametrize("transpose_out", [False, True])
def test_dequantize_bit_exact(cuda_device, mode, rows, cols, transpose_out):
    gs, _ = oq.DEFAULTS[mode]
    if cols % gs:
        pytest.skip("group larger than the row")
    words, scales, biases, gs, bits = _packed(mode, rows, cols, seed=rows + cols)
    # a NaN scale code stays NaN (E8M0 255 / E4M3 0x7F); affine scales are plain bf16
    if mode != "affine":
        scales = scales.clone()
        scales[0, 0] = 0x7F if mode == "nvfp4" else 255
    exp = oq.dequantize(words, scales, biases, mode=mode, group_size=gs, bits=bits)
    got = ops.dequantize(words.to(cuda_device), scales.to(cuda_device),
                         None if biases is None else biases.to(cuda_device), mode=mode,
                         group_size=gs, bits=bits, transpose_out=transpose_out).cpu()
    if transpose_out:
        exp = exp.t()
    assert got.shape == exp.shape
    same = (got == exp) | (torch.isnan(got) & torch.isnan(exp))
    assert bool(same.all()), int((~same).sum())


@pytest.mark.parametrize("mode", ["mxfp8", "nvfp4", "affine"])
@pytest.mark.parametrize("transpose", [True, False])
def test_quantized_linear_matches_oracle(cuda_device, mode, transpose):
    m, n, k = 200, 384, 512
    g = torch.Generator().manual_seed(11)
    w = torch.randn((n, k), generator=g) * 0.05
    src = w if transpose else w.t().contiguous()
    gs, bits = oq.DEFAULTS[mode]
    words, scales, biases = oq.quantize(src, mode=mode, group_size=gs, bits=bits)
    x = normal((m, k), seed=12)
    bias = normal((n,), seed=13, std=0.1)
    exp = oq.quantized_matmul(x, words, scales, biases, mode=mode, group_size=gs, bits=bits,
                              transpose=transpose, bias=bias)
    dev = cuda_device
    got = ops.quantized_linear(x.to(dev), words.to(dev), scales.to(dev),
                               None if biases is None else biases.to(dev), mode=mode,
                               group_size=gs, bits=bits, transpose=transpose, bias=bias.to(dev))
    o, e = got.float().cpu(), exp.float()
    assert float((o - e).abs().max() / e.abs().max()) <= 2e-2
    assert (got.cpu() == exp).float().mean() > 0.9


def _pack_blocks(w, v, transposed):
    """The reference's mxfp8-blocks conversion of every block linear (oracle quantiser): a packed
    checkpoint for the device and the dequantised bf16 weights for the oracle."""
    packed, dequant = dict(w), dict(w)
    bases = ["attn1.to_q", "attn1.to_k", "attn1.to_v", "attn1.to_out", "attn1.to_gate_logits",
             "attn2.to_q", "attn2.to_k", "attn2.to_v", "attn2.to_out", "attn2.to_gate_logits",
             "ff.project_in.proj", "ff.project_out"]
    for i in range(v.blocks):
        for b in bases:
            key = f"transformer_blocks.{i}.{b}"
            wt = w[f"{key}.weight"].float()
            src = wt.t().contiguous() if transposed else wt
            words, scales, _ = oq.quantize(src, mode="mxfp8", group_size=32, bits=8)
            d = oq.dequantize(words, scales, None, mode="mxfp8", group_size=32, bits=8)
            packed[f"{key}.weight"], packed[f"{key}.scales"] = words, scales
            dequant[f"{key}.weight"] = d.t().contiguous() if transposed else d
    return packed, dequant


class _PackedVariant:
    """The variant for the oracle with the reference's packed-linear rounding (matmul rounded to
    bf16, then + bias) on the block linears."""

    packed_blocks = True

    def __init__(self, v):
        self._v = v

    def __getattr__(self, name):
        return getattr(self._v, name)


@pytest.mark.parametrize("quantize", ["mxfp8-blocks", "mxfp8-blocks-pretranspose"])
def test_packed_ltx_block_matches_oracle(cuda_device, quantize):
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=0)
    packed, dequant = _pack_blocks(w, v, quantize.endswith("pretranspose"))
    grid = (3, 4, 8)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=1)
    context = normal((1, 64, v.context_dim), seed=2)
    pos = ref.pixel_coords(ref.patch_grid_bounds(*grid))
    sigma = ref.DISTILLED_STAGE_1_SIGMAS[5]
    expect = ref.forward(dequant, latent, context, sigma, pos, _PackedVariant(v))
    model = LTXVideoTransformer(packed, v, cuda_device, quantize=quantize)
    out = model.run(model.prepare(context, pos), latent.to(cuda_device), sigma).clone()
    o, e = out.float().cpu().flatten(), expect.float().flatten()
    rel_l2 = float((o - e).norm() / e.norm())
    max_rel = float((o - e).abs().max() / e.abs().max())
    cos = float(torch.nn.functional.cosine_similarity(o, e, dim=0))
    assert rel_l2 <= 1e-2 and max_rel <= 2e-2 and cos >= 0.999, (rel_l2, max_rel, cos)


def test_packed_ltx_load_time_conversion(cuda_device):
    """A bf16 checkpoint converted at load (no `.scales` keys) runs and matches the same model
    given the oracle's packing of those weights, bit for bit."""
    v = lcfg.BASELINE_VIDEO.with_blocks(1)
    w = ltx_weights(v, seed=4)
    packed, _ = _pack_blocks(w, v, False)
    grid = (2, 4, 8)
    latent = normal((1, grid[0] * grid[1] * grid[2], v.in_channels), seed=5, device=cuda_device)
    context = normal((1, 32, v.context_dim), seed=6)
    pos = ref.pixel_coords(ref.patch_grid_bounds(*grid))
    a = LTXVideoTransformer(w, v, cuda_device, quantize="mxfp8-blocks")
    b = LTXVideoTransformer(packed, v, cuda_device, quantize="mxfp8-blocks")
    ya = a.run(a.prepare(context, pos), latent, 0.5).clone()
    yb = b.run(b.prepare(context, pos), latent, 0.5).clone()
    torch.cuda.synchronize()
    assert torch.equal(ya, yb)
