"""`kinomlx.kernels.winograd_conv3d.WinogradConv3d` surface (kinomlx/kernels/winograd_conv3d.py:
561-735) on the tcgen05 implicit-GEMM conv.

The reference transforms 6 x 6 output tiles with Winograd F(6x6, 3x3) per temporal tap because
that is what its GPU does fastest; here the same convolution (3 x 3 x 3 taps, one replicated
frame at each temporal end, spatial zero padding 1, fp32 accumulation rounded to bf16, then the
bias added in bf16) runs as one implicit GEMM whose input boxes the TMA unit loads straight from
the unpadded tensor. Same constructor, `supports` and `__call__(x, weight, bias)`; the transient
output-block option is validated as the reference does and has nothing to change here (the
kernel holds no transformed filters).
"""

from __future__ import annotations

import torch

from .. import ops, ops_f32


class WinogradConv3d:
    """Non-causal 3 x 3 x 3 conv of batch-one BTHWC activations with OTHWI weights."""

    def __init__(self, *, transient_output_block: int | None = None) -> None:
        if transient_output_block is not None and (
            transient_output_block <= 0 or transient_output_block % 4
        ):
            raise ValueError("transient Winograd output block must be a positive multiple of four")
        self._transient_output_block = transient_output_block

    @staticmethod
    def supports(x: torch.Tensor, weight: torch.Tensor) -> bool:
        """True when the device conv takes these operands: batch one, 3 x 3 x 3 OTHWI weights of
        the input's dtype (bf16, or fp32 for the parity mode), CUDA tensors, input channels a
        multiple of 64 and output channels a multiple of 8 in bf16."""
        if x.dim() != 5 or weight.dim() != 5 or x.shape[0] != 1:
            return False
        channels = int(x.shape[-1])
        output, taps, kh, kw, weight_channels = (int(value) for value in weight.shape)
        if (taps, kh, kw) != (3, 3, 3) or channels != weight_channels:
            return False
        if not (x.is_cuda and weight.is_cuda) or weight.dtype != x.dtype:
            return False
        if x.dtype == torch.bfloat16:
            return channels % 64 == 0 and output % 8 == 0
        return x.dtype == torch.float32

    def __call__(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
        """Convolve BTHWC with one temporal edge repeat on each side; returns (1, T, H, W, O)."""
        if (
            x.dim() != 5
            or x.shape[0] != 1
            or weight.dim() != 5
            or tuple(weight.shape[1:4]) != (3, 3, 3)
            or x.shape[-1] != weight.shape[-1]
            or x.dtype != weight.dtype
        ):
            raise ValueError("Winograd Conv3d requires batch-one BTHWC and OTHWI 3x3x3 weights")
        if not self.supports(x, weight):
            raise ValueError("the device conv does not take these operands "
                             f"({tuple(x.shape)} {x.dtype}, weight {tuple(weight.shape)})")
        conv = ops.conv3d if x.dtype == torch.bfloat16 else ops_f32.conv3d
        out = conv(x.contiguous(), weight.contiguous(), bias, causal=False)
        return out[None]


__all__ = ["WinogradConv3d"]
