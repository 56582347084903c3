"""Packed-weight formats (affine, mxfp8, mxfp4, nvfp4): the oracle's decoders pinned against
hand-derived code points, the packing round trip, and the product's load-time mxfp8 conversion
against the oracle's (CPU only)."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import quantized as oq
from kinomlx_b200.ltx2 import quantization as qz


def test_e4m3_code_points():
    # S.EEEE.MMM, bias 7: 0x38 = 1.0, 0x7E = 448 (largest), 0x01 = 2^-9 (smallest subnormal),
    # 0x08 = 2^-6 (smallest normal), 0xB8 = -1, 0x7F and 0xFF NaN, 0x00 zero
    got = oq.decode_e4m3(torch.tensor([0x38, 0x7E, 0x01, 0x08, 0xB8, 0x00, 0x3C, 0x30]))
    assert got.tolist() == [1.0, 448.0, 2.0 ** -9, 2.0 ** -6, -1.0, 0.0, 1.5, 0.5]
    assert torch.isnan(oq.decode_e4m3(torch.tensor([0x7F, 0xFF]))).all()


def test_e2m1_and_e8m0_code_points():
    assert oq.decode_e2m1(torch.arange(8)).tolist() == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert oq.decode_e2m1(torch.tensor([0xF, 0x9])).tolist() == [-6.0, -0.5]
    assert oq.decode_e8m0(torch.tensor([127, 128, 126, 254])).tolist() == [1.0, 2.0, 0.5, 2.0 ** 127]
    assert oq.decode_e8m0(torch.tensor([0])).item() == 2.0 ** -127
    assert torch.isnan(oq.decode_e8m0(torch.tensor([255]))).all()


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_unpack_round_trip(bits):
    g = torch.Generator().manual_seed(3)
    codes = torch.randint(0, 2 ** bits, (5, 64), generator=g)
    words = oq.pack(codes, bits)
    assert words.dtype == torch.int32 and words.shape == (5, 64 * bits // 32)
    assert torch.equal(oq.unpack(words, bits), codes)
    # element 1 of a 4-bit row sits in bits 4..7 of word 0 (little-endian within the word)
    if bits == 4:
        one = torch.zeros((1, 8), dtype=torch.int64)
        one[0, 1] = 0xA
        assert oq.pack(one, 4).item() == 0xA0


@pytest.mark.parametrize("mode", ["affine", "mxfp8", "mxfp4", "nvfp4"])
def test_quantize_dequantize_error(mode):
    """Synthetic quantisation then dequantisation stays within each format's resolution."""
    g = torch.Generator().manual_seed(5)
    w = torch.randn((16, 256), generator=g) * 0.05
    gs, bits = oq.DEFAULTS[mode]
    words, scales, biases = oq.quantize(w, mode=mode, group_size=gs, bits=bits)
    d = oq.dequantize(words, scales, biases, mode=mode, group_size=gs, bits=bits).float()
    rel = float((d - w).norm() / w.norm())
    bound = {"affine": 0.12, "mxfp8": 0.05, "mxfp4": 0.2, "nvfp4": 0.15}[mode]
    assert rel < bound, rel


def test_product_mxfp8_conversion_matches_oracle():
    """The load-time converter (torch float8 rounding) gives the oracle's codes and scales."""
    g = torch.Generator().manual_seed(7)
    w = (torch.randn((32, 128), generator=g) * 0.03).to(torch.bfloat16)
    words, scales = qz.quantize_mxfp8(w.float())
    ow, os_, _ = oq.quantize(w.float(), mode="mxfp8", group_size=32, bits=8)
    assert torch.equal(scales, os_)
    assert torch.equal(words, ow)
    d = oq.dequantize(words, scales, None, mode="mxfp8", group_size=32, bits=8)
    assert float((d.float() - w.float()).abs().max()) <= float(w.float().abs().max()) * 2 ** -3


def test_quantized_matmul_orientations():
    """x @ W^T from the (out, in) packing equals x @ W from the packing of weight.T."""
    g = torch.Generator().manual_seed(9)
    w = torch.randn((64, 128), generator=g) * 0.05
    x = torch.randn((4, 128), generator=g).to(torch.bfloat16)
    a = oq.quantize(w, mode="mxfp8", group_size=32, bits=8)
    ya = oq.quantized_matmul(x, a[0], a[1], None, mode="mxfp8", group_size=32, bits=8, transpose=True)
    b = oq.quantize(w.t().contiguous(), mode="mxfp8", group_size=32, bits=8)
    yb = oq.quantized_matmul(x, b[0], b[1], None, mode="mxfp8", group_size=32, bits=8, transpose=False)
    assert ya.shape == yb.shape == (4, 64)
    assert math.isclose(float((ya.float() - yb.float()).norm() / ya.float().norm()), 0.0, abs_tol=0.08)
