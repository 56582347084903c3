"""`kinomlx.kernels.mpp_linear` surface (kinomlx/kernels/mpp_linear.py:340-632) on tcgen05.

The reference converts bf16 operands to power-of-two-scaled fp16 because the M1 has no bf16
arithmetic; the B200 multiplies bf16 natively with fp32 accumulation, so `prepare`, `restore`
and `fp16_operand` are identities that keep the reference's call shape.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import torch

from .. import ops

MIN_ROWS = 1
MIN_WIDTH = 8
_DTYPES = (torch.bfloat16,)
_enabled = True


class Operand(NamedTuple):
    values: torch.Tensor
    peak: torch.Tensor | None


def set_enabled(enabled: bool) -> None:
    global _enabled
    _enabled = bool(enabled)


def enabled() -> bool:
    return _enabled


def fp16_operand(value: torch.Tensor) -> Operand:
    return Operand(value, None)


def prepare(weight: torch.Tensor) -> Operand:
    return Operand(weight, None)


def restore(prepared: Operand) -> torch.Tensor:
    return prepared.values


def supports(rows: int, k: int, n: int, *, transposed: bool, dtype: torch.dtype) -> bool:
    """(out, in) weights, widths multiples of 8 (TMA row alignment), bf16."""
    return transposed and dtype in _DTYPES and rows >= 1 and k % 8 == 0 and n % 8 == 0


def available(*, transposed: bool, bias: bool, dtype: torch.dtype = torch.bfloat16) -> bool:
    return transposed and dtype in _DTYPES


def _weight(weight):
    return weight.values if isinstance(weight, Operand) else weight


def applies(value, weight, bias, *, transposed: bool) -> bool:
    w = _weight(weight)
    if not _enabled or value.dim() < 2 or w.dim() != 2 or not value.is_cuda:
        return False
    if value.dtype not in _DTYPES or w.dtype != value.dtype:
        return False
    n, inner = w.shape if transposed else w.shape[::-1]
    if inner != value.shape[-1]:
        return False
    if bias is not None and (bias.dtype != value.dtype or tuple(bias.shape) != (n,)):
        return False
    rows = math.prod(value.shape[:-1])
    return supports(rows, value.shape[-1], n, transposed=transposed, dtype=value.dtype)


def linear(value, weight, bias, *, transposed: bool, operand: Operand | None = None):
    """addmm(bias, value, weight.T) for an (out, in) weight: fp32 accumulation, bias added to the
    fp32 sum, one rounding (kinomlx/kernels/mpp_linear.py:469-506)."""
    w = _weight(weight)
    if not transposed:
        raise ValueError("the B200 GEMM takes (out, in) weights (transposed=True)")
    if w.dtype != value.dtype:
        raise ValueError(f"linear multiplies a {value.dtype} input by a weight of that dtype, not {w.dtype}")
    rows = math.prod(value.shape[:-1])
    if not supports(rows, value.shape[-1], w.shape[0], transposed=True, dtype=value.dtype):
        raise ValueError(
            f"the B200 GEMM does not take a {rows} x {value.shape[-1]} by {value.shape[-1]} x "
            f"{w.shape[0]} {value.dtype} product"
        )
    flat = value.reshape(rows, value.shape[-1])
    return ops.linear(flat, w.contiguous(), bias=bias).reshape(*value.shape[:-1], w.shape[0])


_ONES: dict[tuple, torch.Tensor] = {}


def linear_rows(value, weight, bias=None, *, residual=None):
    """residual + addmm(bias, value, weight.T) with the product rounded before the residual add
    (kinomlx/kernels/mpp_linear.py:592-611). The add runs in the GEMM's epilogue: the gated
    residual form with a gate of ones, residual + round(1 * round(acc + bias)), rounded once
    more at the store, is that sum."""
    if residual is None:
        return linear(value, weight, bias, transposed=True)
    w = _weight(weight)
    n = w.shape[0]
    if residual.dtype != value.dtype or tuple(residual.shape) != (*value.shape[:-1], n):
        raise ValueError(f"the residual must be a {value.dtype} {(*value.shape[:-1], n)} tensor")
    rows = math.prod(value.shape[:-1])
    if w.dtype != value.dtype or not supports(rows, value.shape[-1], n, transposed=True,
                                              dtype=value.dtype):
        raise ValueError(
            f"the B200 GEMM does not take a {rows} x {value.shape[-1]} by {value.shape[-1]} x "
            f"{n} {value.dtype} product")
    key = (value.device, n, value.dtype)
    if key not in _ONES:
        _ONES[key] = torch.ones((1, n), device=value.device, dtype=value.dtype)
    res = residual.reshape(rows, n).contiguous()
    out = torch.empty_like(res)
    ops.linear(value.reshape(rows, value.shape[-1]), w.contiguous(), out, bias=bias,
               kind=ops.EPI_GATED_RESIDUAL, residual=res, gate=_ONES[key])
    return out.reshape(*value.shape[:-1], n)
