"""Exact 3-D neighborhood attention restated on the CPU (test oracle; nothing else may import it).

Follows kinomlx/models/ltx2/kernels/neighborhood_attention.py:1-221, the attention of the LTX-2.5
diffusion video decoder: every query of a (T, H, W) token grid attends to the KT x KH x KW keys
of its window, which keeps its full size at the grid edges by shifting inward (on an axis of
length L the window of position i starts at clamp(i - K // 2, 0, L - K)). Operands are
token-major (batch, T, H, W, heads, 64) fp16 with the queries already scaled; scores, softmax
and output accumulate in fp32 and the output is rounded to fp16 once.

Also restated: which calls the reference's kernels take (`supports`, `applies`, `launch_fits`,
neighborhood_attention.py:99-167), a host contract (odd window inside the grid, a grid large
enough for one of its two kernels' key boxes, a launch grid inside MLX's signed 32-bit
dimensions); callers keep a masked dense attention where it is false.

Pinned in tests/test_neighborhood_attention_oracle.py against the reference's own tests
(tests/models/ltx2/test_neighborhood_attention.py).
"""

from __future__ import annotations

import math

import torch

HEAD_DIM = 64
KEY_RUN = 16
THREADS = 128
RUN_TILES = {(3, 7, 7): (2, 2, 8), (3, 5, 5): (1, 4, 8), (11, 11, 11): (4, 2, 4)}
PATCH_FRAMES = 8
GRID_LIMIT = 2**31 - 1


def window_starts(length: int, size: int) -> torch.Tensor:
    """First key index of each position's window on one axis."""
    return torch.clamp(torch.arange(length) - size // 2, 0, length - size)


def window_keys(grid: tuple[int, int, int], window: tuple[int, int, int]) -> torch.Tensor:
    """(tokens, KT*KH*KW) raster indices of every query's window keys."""
    gt, gh, gw = grid
    idx = [window_starts(n, k)[:, None] + torch.arange(k)[None, :] for n, k in zip(grid, window)]
    keys = (idx[0][:, None, None, :, None, None] * (gh * gw)
            + idx[1][None, :, None, None, :, None] * gw
            + idx[2][None, None, :, None, None, :])
    return keys.reshape(gt * gh * gw, math.prod(window))


def neighborhood_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                           window: tuple[int, int, int]) -> torch.Tensor:
    """Attention of each scaled query over its window's keys: fp32 scores and softmax, the
    output rounded to the inputs' dtype."""
    batch, gt, gh, gw, heads, dim = q.shape
    tokens = gt * gh * gw
    keys = window_keys((gt, gh, gw), window)
    out = torch.empty((batch, tokens, heads, dim), dtype=torch.float32)
    for b in range(batch):
        qf, kf, vf = (x[b].reshape(tokens, heads, dim).float() for x in (q, k, v))
        for start in range(0, tokens, 256):
            sel = keys[start : start + 256]
            scores = torch.einsum("nhd,nkhd->nhk", qf[start : start + 256], kf[sel])
            out[b, start : start + 256] = torch.einsum("nhk,nkhd->nhd", torch.softmax(scores, -1), vf[sel])
    return out.reshape(q.shape).to(q.dtype)


def run_tile(window: tuple[int, int, int]) -> tuple[int, int, int]:
    """Query block of the reference's `runs` kernel (neighborhood_attention.py:99-104)."""
    if window in RUN_TILES:
        return RUN_TILES[window]
    return (4, 2, 4) if window[2] > 9 else (4, 1, 8)


def _patches_fit(window, grid) -> bool:
    kt, kh, kw = window
    return window == (11, 11, 11) and grid[0] >= PATCH_FRAMES + kt - 1 and grid[1] >= kh + 1 \
        and grid[2] >= kw + 1


def _runs_fit(window, grid) -> bool:
    qt, qh, qw = run_tile(window)
    kt, kh, kw = window
    return qw + kw - 1 <= KEY_RUN and grid[0] >= qt + kt - 1 and grid[1] >= qh + kh - 1 \
        and grid[2] >= KEY_RUN


def _launch_tiles(window, grid) -> int:
    gt, gh, gw = grid
    if _patches_fit(window, grid):
        return -(-gt // PATCH_FRAMES) * -(-gh // 2) * -(-gw // 2)
    qt, qh, qw = run_tile(window)
    return -(-gt // qt) * -(-gh // qh) * -(-gw // qw)


def launch_fits(grid, window) -> bool:
    """128 threads per 32-query block within a signed 32-bit grid (neighborhood_attention.py:137-141)."""
    return _launch_tiles(window, grid) * THREADS <= GRID_LIMIT


def supports(shape: tuple[int, ...], window) -> bool:
    """neighborhood_attention.py:144-157."""
    if len(shape) != 6 or shape[-1] != HEAD_DIM or math.prod(shape) <= 0:
        return False
    grid = (int(shape[1]), int(shape[2]), int(shape[3]))
    if any(size % 2 == 0 or size < 1 for size in window):
        return False
    if any(size > length for size, length in zip(window, grid)):
        return False
    if not (_patches_fit(window, grid) or _runs_fit(window, grid)):
        return False
    return launch_fits(grid, window)


def applies(q_shape, k_shape, v_shape, dtypes, *, window) -> bool:
    """Matching fp16 operands of a supported shape (neighborhood_attention.py:160-167); shapes
    and dtypes only, so calls past 2**31 elements can be asked about without arrays."""
    if tuple(k_shape) != tuple(q_shape) or tuple(v_shape) != tuple(q_shape):
        return False
    if any(dt != torch.float16 for dt in dtypes):
        return False
    return supports(tuple(int(s) for s in q_shape), window)
