"""`kinomlx.models.ltx2.kernels.sol_attention` surface (kinomlx/models/ltx2/kernels/
sol_attention.py:98-275): Sol-Attn routed sparse attention on the tcgen05 kernels.

Same names, arguments and refusals as the reference; `sol_attention` is one call into
libkino_b200.so (preparation, routing and attention on the device; no CPU path). `morton_order`
is host index arithmetic, computed once per latent grid.
"""

from __future__ import annotations

import math

import torch

from .. import ops

BLOCK = 64
HEAD_DIM = 128
_WORD_BITS = 32
_SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)
MAX_BLOCKS = 512  # the device kernel keeps each query block's routing row in 16 mask words
QUERY_BLOCKS_PER_CTA = 2  # the attention kernel's 128-row query tile covers two blocks


def block_count(tokens: int) -> int:
    """The number of 64-token blocks covering `tokens`."""
    return (tokens + BLOCK - 1) // BLOCK


def morton_order(frames: int, height: int, width: int, *, tokens: int | None = None) -> torch.Tensor:
    """Raster indices of an (F, H, W) token grid in 3-D Morton order: bit i of the frame, row and
    column goes to bits 3i, 3i + 1 and 3i + 2 of the key; tokens past the grid (appended
    conditioning) keep their order after it (sol_attention.py:106-136). int32, on the host."""
    if min(frames, height, width) <= 0:
        raise ValueError(f"Morton order needs a positive grid, got {frames}x{height}x{width}")
    grid = frames * height * width
    total = grid if tokens is None else tokens
    if total < grid:
        raise ValueError(f"{total} tokens cannot hold a {frames}x{height}x{width} grid")
    bits = max(frames, height, width).bit_length()

    def spread(size: int, shift: int) -> torch.Tensor:
        index = torch.arange(size, dtype=torch.int64)
        key = torch.zeros_like(index)
        for bit in range(bits):
            key |= ((index >> bit) & 1) << (3 * bit + shift)
        return key

    keys = (spread(frames, 0)[:, None, None] | spread(height, 1)[None, :, None]
            | spread(width, 2)[None, None, :]).reshape(-1)
    order = torch.argsort(keys, stable=True)
    if total > grid:
        order = torch.cat([order, torch.arange(grid, total)])
    return order.to(torch.int32)


def _check_inputs(q, k, v, heads: int, order) -> None:
    if q.dtype not in _SUPPORTED_DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(
            f"Sol attention needs float16 or bfloat16 q, k and v, got {q.dtype}, {k.dtype}, {v.dtype}")
    if q.dim() != 2 or q.shape[1] != heads * HEAD_DIM or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(
            f"Sol attention needs (tokens, {heads} * {HEAD_DIM}) q, k and v, got "
            f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if tuple(order.shape) != (q.shape[0],):
        raise ValueError(f"the token order must hold one index per token, got {tuple(order.shape)}")
    if block_count(q.shape[0]) > MAX_BLOCKS:
        raise ValueError(f"the device Sol attention supports at most {MAX_BLOCKS} blocks of 64 tokens")


def _device_order(order: torch.Tensor, device: torch.device) -> torch.Tensor:
    return order.to(device=device, dtype=torch.int32).contiguous()


def sol_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, tau: float,
                  order: torch.Tensor) -> torch.Tensor:
    """Sol-Attn of (tokens, heads * 128) inputs routed in `order`; the output comes back in the
    inputs' order and dtype (sol_attention.py:219-272)."""
    if not math.isfinite(tau):
        raise ValueError(f"Sol attention tau must be finite, got {tau}")
    _check_inputs(q, k, v, heads, order)
    return ops.sol_attention(q, k, v, heads=heads, tau=tau, order=_device_order(order, q.device))


def routed_blocks(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, tau: float,
                  order: torch.Tensor) -> torch.Tensor:
    """The (heads, blocks, blocks) bool routing of one `sol_attention` call as the device
    computed it: entry (h, a, b) is True when query block a attends exactly to key block b."""
    _check_inputs(q, k, v, heads, order)
    blocks = block_count(q.shape[0])
    words = (blocks + _WORD_BITS - 1) // _WORD_BITS
    bits = torch.empty((heads, blocks, words), device=q.device, dtype=torch.int32)
    ops.sol_attention(q, k, v, heads=heads, tau=tau, order=_device_order(order, q.device),
                      routes=bits)
    shifts = torch.arange(_WORD_BITS, device=q.device, dtype=torch.int32)
    flags = (bits[..., None] >> shifts) & 1
    return flags.reshape(heads, blocks, words * _WORD_BITS)[..., :blocks].bool()


__all__ = ["BLOCK", "HEAD_DIM", "block_count", "morton_order", "routed_blocks", "sol_attention"]
