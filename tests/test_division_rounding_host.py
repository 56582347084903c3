"""The divide-free rounding of the PixelNorm kernels (kino_common.cuh, div_round_bf16), checked
on the CPU with numpy's correctly rounded fp32 arithmetic: q = a * r with r within 1 ulp of 1/b,
rounded to bf16, equals bf16(fp32(a / b)) whenever q's low 16 bits lie outside the window around
the half-way pattern 0x8000 that sends an element to the IEEE division instead. Millions of
random operands over many binades, reciprocals exact and perturbed by one ulp either way."""

from __future__ import annotations

import numpy as np


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even) and return the 16-bit patterns."""
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)


def _check(a: np.ndarray, b: np.ndarray, r: np.ndarray, window: int) -> int:
    q = (a * r).astype(np.float32)
    low = q.view(np.uint32) & 0xFFFF
    fast = ((low - (0x8000 - window)) & 0xFFFFFFFF) > 2 * window
    exact = (a / b).astype(np.float32)
    mismatch = fast & (bf16_bits(q) != bf16_bits(exact))
    return int(mismatch.sum())


def test_reciprocal_product_rounds_like_the_quotient():
    rng = np.random.default_rng(7)
    n = 2_000_000
    a = (rng.standard_normal(n) * np.exp2(rng.integers(-20, 20, n))).astype(np.float32)
    b = np.abs(rng.standard_normal(n) * np.exp2(rng.integers(-10, 10, n))).astype(np.float32) + \
        np.float32(1e-4)
    r = (np.float32(1.0) / b).astype(np.float32)  # correctly rounded
    assert _check(a, b, r, 4) == 0
    # an approximate reciprocal within one ulp (the SiLU's rcp.approx) needs the wider window
    for step in (-1, 1):
        rp = (r.view(np.uint32).astype(np.int64) + step).astype(np.uint32).view(np.float32)
        assert _check(a, b, rp, 8) == 0


def test_window_is_needed():
    """Without the fallback window the product does differ from the quotient's rounding."""
    rng = np.random.default_rng(11)
    n = 2_000_000
    a = rng.standard_normal(n).astype(np.float32)
    b = (np.abs(rng.standard_normal(n)) + 0.5).astype(np.float32)
    r = (np.float32(1.0) / b).astype(np.float32)
    rp = (r.view(np.uint32) + 1).view(np.float32)
    assert _check(a, b, rp, 0) > 0
