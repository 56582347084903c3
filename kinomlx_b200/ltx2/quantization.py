"""Packed block linears of the LTX-2 transformer (the reference's `transformer_quantize` modes).

The reference converts the block linears of every transformer block (attention q/k/v/out/gate
projections and the feed-forward in/out projections, kinomlx/models/ltx2/weights/tensors.py:20-46)
to MLX mxfp8 (E4M3 codes with an E8M0 scale per 32 inputs) when `transformer_quantize` is
`mxfp8-blocks`, or packs `weight.T` (scales per 32 outputs) for `mxfp8-blocks-pretranspose`
(weights/schema.py:13-18, weights/quantization.py:17-43), and runs them through
`mx.quantized_matmul`. Here a packed linear keeps its codes and scales in HBM (half the bytes of
bf16) and is dequantised into a bf16 scratch buffer immediately before its tcgen05 GEMM, which
multiplies with fp32 accumulation as the reference's quantized matmul does.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops

MODES = ("off", "mxfp8-blocks", "mxfp8-blocks-pretranspose")
GROUP, BITS = 32, 8  # mxfp8 (kinomlx/models/ltx2/weights/tensors.py:185-203)


@dataclass
class PackedWeight:
    """One packed (out, in) linear weight: codes as 32-bit words and E8M0 scale codes; `transposed`
    means the reference's pretransposed packing of weight.T (along the output dimension)."""

    words: torch.Tensor
    scales: torch.Tensor
    out_features: int
    in_features: int
    transposed: bool

    def dequantize_into(self, dst: torch.Tensor) -> torch.Tensor:
        """Write the bf16 (out, in) weight into `dst` (a view of that shape)."""
        return ops.dequantize(self.words, self.scales, None, mode="mxfp8", group_size=GROUP,
                              bits=BITS, transpose_out=self.transposed, out=dst)


def quantize_mxfp8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Checkpoint conversion (load time, not on the step): a (rows, cols) weight -> (words, scales)
    in MLX's mxfp8 layout along the last axis. Shared exponent per 32 values: floor(log2(amax))
    minus the E4M3 maximum exponent 8 (OCP Microscaling v1.0), elements rounded to nearest-even
    E4M3 after saturating to +-448."""
    rows, cols = w.shape
    if cols % GROUP:
        raise ValueError("mxfp8 packs rows in groups of 32")
    g = w.float().reshape(rows, cols // GROUP, GROUP)
    amax = g.abs().amax(-1).clamp_min(2.0 ** -126)
    e = (torch.frexp(amax).exponent - 1 - 8).clamp(-127, 127)  # floor(log2(amax)) - 8, exactly
    y = torch.ldexp(g, (-e).unsqueeze(-1)).clamp(-448.0, 448.0)  # exact division by 2^e
    codes = y.to(torch.float8_e4m3fn).view(torch.uint8).reshape(rows, cols).contiguous()
    words = codes.view(torch.int32)  # four codes per little-endian word
    scales = (e + 127).to(torch.uint8).contiguous()
    return words, scales


def pack_linear(weight: torch.Tensor, *, transposed: bool, device: torch.device) -> PackedWeight:
    """A bf16 (out, in) weight -> its packed form on `device` (the reference's conversion)."""
    out_f, in_f = weight.shape
    src = weight.t() if transposed else weight
    words, scales = quantize_mxfp8(src.to(device, torch.float32).contiguous())
    return PackedWeight(words, scales, out_f, in_f, transposed)


def packed_from_checkpoint(weights: dict[str, torch.Tensor], base: str, *, transposed: bool,
                           device: torch.device) -> PackedWeight:
    """`base.weight` already packed (int32/uint32 words) with `base.scales`, or a float weight
    converted here."""
    w = weights[f"{base}.weight"]
    if f"{base}.scales" in weights:
        words = w.to(device).contiguous().view(torch.int32)
        scales = weights[f"{base}.scales"].to(device, torch.uint8).contiguous()
        rows, cols = words.shape[0], words.shape[1] * 4
        out_f, in_f = (cols, rows) if transposed else (rows, cols)
        return PackedWeight(words, scales, out_f, in_f, transposed)
    return pack_linear(w, transposed=transposed, device=device)


class PackedGroup:
    """Packed weights that one GEMM uses stacked by output rows (the fused [v | q | k] and
    [k | v] projections): dequantised one after another into consecutive rows of the scratch."""

    def __init__(self, parts: list[PackedWeight]):
        self.parts = parts
        self.in_features = parts[0].in_features
        self.out_features = sum(p.out_features for p in parts)
        if any(p.in_features != self.in_features for p in parts):
            raise ValueError("stacked packed weights need one input width")

    def dequantize(self, scratch: torch.Tensor) -> torch.Tensor:
        """The bf16 (out, in) stacked weight in `scratch` (a flat bf16 buffer)."""
        need = self.out_features * self.in_features
        if scratch.numel() < need:
            raise ValueError("dequantisation scratch too small")
        w = scratch[:need].view(self.out_features, self.in_features)
        r = 0
        for p in self.parts:
            p.dequantize_into(w[r : r + p.out_features])
            r += p.out_features
        return w
