"""Group-quantised weights of the reference's packed linears, restated on the CPU (test oracle).

The reference stores LTX block linears packed (kinomlx/models/ltx2/weights/quantization.py:17-43:
`mx.quantized_matmul(value, weight, scales, biases, transpose=False, group_size, bits, mode)` for
weights packed from `weight.T`; `nn.QuantizedLinear` for the plain orientation) in four modes with
the defaults of kinomlx/models/ltx2/weights/tensors.py:185-203: affine (group 64, 4 bits),
mxfp8 (group 32, 8 bits), mxfp4 (group 32, 4 bits) and nvfp4 (group 16, 4 bits). The arithmetic
lives in MLX (`mlx>=0.32.4`, pyproject.toml:28), which is not vendored under the reference, so
this module restates the published formats instead:

  * packing: `bits`-bit codes along the last axis, little-endian inside uint32 words (element i of
    a row in word i * bits // 32 at bit (i * bits) % 32), 32 // bits codes per word;
  * affine: w = scale * q + bias per group of `group_size` codes, q unsigned, scale and bias in the
    weight's dtype (MLX affine group quantisation);
  * mxfp8 / mxfp4: OCP Microscaling Formats v1.0 -- E4M3 (bias 7, no infinities, S.1111.111 is
    NaN) or E2M1 (bias 1, values 0, 0.5, 1, 1.5, 2, 3, 4, 6) elements times a shared E8M0 scale
    2^(e - 127) per group of 32 (e = 255 is NaN);
  * nvfp4: E2M1 elements times an E4M3 scale per group of 16.

Dequantisation is exact in fp32 for the three float modes (a small-mantissa element times a power
of two or an E4M3 scale) and is one fp32 fma for affine; the result is rounded to bf16 once. The
reference's quantised matmul multiplies bf16 activations by these dequantised weights with fp32
accumulation, so `quantized_matmul` below is the plain matmul of the dequantised weight.

Parity: no golden vectors for these formats exist in the reference (its tests call MLX's own
`mx.quantize`), so this restatement is **parity unpinned** beyond the format definitions; the
CPU tests pin the decoders against hand-derived code points.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).
"""

from __future__ import annotations

import torch

MODES = {"affine": 0, "mxfp8": 1, "mxfp4": 2, "nvfp4": 3}
DEFAULTS = {"affine": (64, 4), "mxfp8": (32, 8), "mxfp4": (32, 4), "nvfp4": (16, 4)}


def decode_e4m3(code: torch.Tensor) -> torch.Tensor:
    """E4M3 byte -> float32 (sign, 4-bit exponent with bias 7, 3-bit mantissa, no infinities)."""
    c = code.to(torch.int32) & 0xFF
    sign = torch.where((c & 0x80) != 0, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = (c & 0x7).to(torch.float32)
    normal = (1.0 + m / 8.0) * torch.pow(2.0, (e - 7).to(torch.float32))
    sub = m / 8.0 * 2.0 ** -6
    v = torch.where(e == 0, sub, normal) * sign
    return torch.where((c & 0x7F) == 0x7F, torch.full_like(v, float("nan")), v)


def decode_e2m1(code: torch.Tensor) -> torch.Tensor:
    """E2M1 nibble -> float32 (sign, 2-bit exponent with bias 1, 1-bit mantissa)."""
    c = code.to(torch.int32) & 0xF
    table = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    v = table[c & 0x7]
    return torch.where((c & 0x8) != 0, -v, v)


def decode_e8m0(code: torch.Tensor) -> torch.Tensor:
    """E8M0 byte -> float32 2^(e - 127); 255 is NaN."""
    e = code.to(torch.int32) & 0xFF
    v = torch.pow(2.0, (e - 127).to(torch.float64)).to(torch.float32)
    return torch.where(e == 255, torch.full_like(v, float("nan")), v)


def unpack(words: torch.Tensor, bits: int) -> torch.Tensor:
    """(..., n_words) uint32-valued int64/int32 words -> (..., n_words * 32 // bits) codes."""
    if 32 % bits:
        raise ValueError("only bit widths that divide 32 are packed whole into words")
    per = 32 // bits
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, dtype=torch.int64) * bits
    codes = (w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    return codes.reshape(*words.shape[:-1], words.shape[-1] * per)


def pack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Inverse of `unpack`: (..., n) codes -> (..., n * bits // 32) words as int32."""
    per = 32 // bits
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], codes.shape[-1] // per, per)
    shifts = torch.arange(per, dtype=torch.int64) * bits
    w = (c << shifts).sum(-1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def dequantize(words: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor | None, *,
               mode: str, group_size: int, bits: int) -> torch.Tensor:
    """Packed (rows, cols * bits / 32) words, per-group scales (and affine biases) of shape
    (rows, cols / group_size) -> the bf16 (rows, cols) weight."""
    codes = unpack(words, bits)
    rows, cols = codes.shape
    g = cols // group_size
    if mode == "affine":
        s = scales.float().repeat_interleave(group_size, -1)
        b = biases.float().repeat_interleave(group_size, -1)
        # one fp32 fma per element, rounded once
        w = torch.addcmul(b.double(), s.double(), codes.double()).float()
    else:
        elem = decode_e4m3(codes) if mode == "mxfp8" else decode_e2m1(codes)
        sc = decode_e4m3(scales) if mode == "nvfp4" else decode_e8m0(scales)
        w = elem * sc.reshape(rows, g).repeat_interleave(group_size, -1)
    return w.to(torch.bfloat16)


def quantized_matmul(x: torch.Tensor, words: torch.Tensor, scales: torch.Tensor,
                     biases: torch.Tensor | None, *, mode: str, group_size: int, bits: int,
                     transpose: bool, bias: torch.Tensor | None = None) -> torch.Tensor:
    """x @ W^T (transpose, packed (N, K) along K) or x @ W (packed (K, N) along N, the
    pretransposed form), fp32 accumulation of bf16 operands, rounded once, then + bias in bf16
    (kinomlx/models/ltx2/weights/quantization.py:26-43)."""
    w = dequantize(words, scales, biases, mode=mode, group_size=group_size, bits=bits)
    wt = w if transpose else w.t()
    y = (x.float() @ wt.float().t()).to(torch.bfloat16)
    return y + bias if bias is not None else y


# --------------------------------------------------------------------- synthetic quantisation
_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _nearest_code(x: torch.Tensor, grid: torch.Tensor) -> torch.Tensor:
    """Index of the nearest value of the increasing non-negative `grid` to |x|; a tie goes to
    the even index (round half to even on the code)."""
    a = x.abs().contiguous()
    hi = torch.searchsorted(grid, a).clamp(1, grid.numel() - 1)
    lo = hi - 1
    dl, dh = a - grid[lo], grid[hi] - a
    pick_hi = (dh < dl) | ((dh == dl) & (hi % 2 == 0))
    idx = torch.where(pick_hi, hi, lo)
    return torch.where(a >= grid[-1], torch.full_like(idx, grid.numel() - 1), idx)


def _e4m3_grid() -> torch.Tensor:
    return decode_e4m3(torch.arange(0, 0x7F))  # non-negative finite codes 0..126


def quantize(w: torch.Tensor, *, mode: str, group_size: int, bits: int):
    """A float (rows, cols) weight -> (words int32, scales, biases or None) in the packed layout
    above. Only used to make synthetic quantised weights for tests and benchmarks; the scale
    choice follows the OCP MX recipe (shared exponent floor(log2(amax)) - emax of the element
    format) and, for affine, min/max over the group."""
    rows, cols = w.shape
    g = w.float().reshape(rows, cols // group_size, group_size)
    if mode == "affine":
        lo, hi = g.min(-1).values, g.max(-1).values
        scale = ((hi - lo) / (2 ** bits - 1)).clamp_min(1e-8).to(torch.bfloat16)
        bias = lo.to(torch.bfloat16)
        q = torch.round((g - bias.float().unsqueeze(-1)) / scale.float().unsqueeze(-1))
        q = q.clamp(0, 2 ** bits - 1).to(torch.int64).reshape(rows, cols)
        return pack(q, bits), scale, bias
    amax = g.abs().amax(-1).clamp_min(1e-30)
    if mode == "nvfp4":
        grid = _e4m3_grid()
        sc_code = _nearest_code(amax / 6.0, grid)  # E4M3 scale per 16
        sc = grid[sc_code].clamp_min(2.0 ** -9)
        sc_code = _nearest_code(sc, grid)
        y = g / sc.unsqueeze(-1)
        elem_grid, sign_bit = _E2M1, 8
        scales = sc_code.to(torch.uint8)
    else:
        emax = 8 if mode == "mxfp8" else 2
        e = torch.frexp(amax).exponent.to(torch.int64) - 1 - emax  # floor(log2(amax)) - emax
        e = e.clamp(-127, 127)
        y = torch.ldexp(g, (-e).unsqueeze(-1))  # exact division by 2^e
        elem_grid = _e4m3_grid() if mode == "mxfp8" else _E2M1
        sign_bit = 0x80 if mode == "mxfp8" else 8
        scales = (e + 127).to(torch.uint8)
    y = y.clamp(-float(elem_grid.max()), float(elem_grid.max()))
    code = _nearest_code(y, elem_grid) | torch.where(y < 0, sign_bit, 0)
    code = torch.where((code & ~sign_bit) == 0, torch.zeros_like(code), code)  # +0 for zeros
    return pack(code.reshape(rows, cols), bits), scales, None


def default_group(mode: str) -> tuple[int, int]:
    """(group_size, bits) defaults per mode (kinomlx/models/ltx2/weights/tensors.py:185-203)."""
    return DEFAULTS[mode]

