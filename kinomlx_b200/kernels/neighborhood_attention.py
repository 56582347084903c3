"""The reference's neighborhood-attention surface (kinomlx/models/ltx2/kernels/
neighborhood_attention.py) over the B200 kernel `kino_neighborhood_attention`.

Exact 3-D neighborhood attention of the LTX-2.5 diffusion video decoder: every query of a
(T, H, W) grid attends to the KT x KH x KW keys of its window, which keeps its full size at the
grid edges by shifting inward (on an axis of length L the window of position i starts at
clamp(i - K // 2, 0, L - K)). Operands are token-major (batch, T, H, W, heads, 64) fp16 with the
queries already scaled.

`supports`, `applies`, `launch_fits` and `run_tile` keep the reference's host contract
(neighborhood_attention.py:99-167), so a caller takes the kernel path for exactly the calls it
took there and keeps its masked fallback elsewhere. The device kernel itself is wider: any odd
window no larger than the grid (`kinomlx_b200.ops.neighborhood_attention`).
"""

from __future__ import annotations

import math

import torch

from .. import ops

HEAD_DIM = 64
_KEY_RUN = 16
_THREADS = 128
_RUN_TILES = {(3, 7, 7): (2, 2, 8), (3, 5, 5): (1, 4, 8), (11, 11, 11): (4, 2, 4)}
_PATCH_FRAMES = 8
_GRID_LIMIT = 2**31 - 1

Grid = tuple[int, int, int]

_enabled = True


def set_enabled(enabled: bool) -> None:
    """Switch the kernel path on or off (`applies` is false while it is off)."""
    global _enabled
    _enabled = bool(enabled)


def enabled() -> bool:
    return _enabled


def run_tile(window: Grid) -> Grid:
    """The query block the reference's `runs` kernel takes for `window` (:99-104)."""
    if tuple(window) in _RUN_TILES:
        return _RUN_TILES[tuple(window)]
    return (4, 2, 4) if window[2] > 9 else (4, 1, 8)


def _patches_fit(window: Grid, grid: Grid) -> bool:
    kt, kh, kw = window
    return tuple(window) == (11, 11, 11) and grid[0] >= _PATCH_FRAMES + kt - 1 \
        and grid[1] >= kh + 1 and grid[2] >= kw + 1


def _runs_fit(window: Grid, grid: Grid) -> bool:
    qt, qh, qw = run_tile(window)
    kt, kh, kw = window
    return qw + kw - 1 <= _KEY_RUN and grid[0] >= qt + kt - 1 and grid[1] >= qh + kh - 1 \
        and grid[2] >= _KEY_RUN


def _launch_tiles(window: Grid, grid: Grid) -> int:
    gt, gh, gw = grid
    if _patches_fit(window, grid):
        return -(-gt // _PATCH_FRAMES) * -(-gh // 2) * -(-gw // 2)
    qt, qh, qw = run_tile(window)
    return -(-gt // qt) * -(-gh // qh) * -(-gw // qw)


def launch_fits(grid: Grid, window: Grid) -> bool:
    """The reference's launch-size bound (:137-141)."""
    return _launch_tiles(window, grid) * _THREADS <= _GRID_LIMIT


def supports(shape: tuple[int, ...], window: Grid) -> bool:
    """Whether the kernel path takes (batch, T, H, W, heads, 64) arrays of `shape` with
    `window` (:144-157): an odd window inside the grid, a grid large enough for one of the
    reference kernels' key boxes, a launch within its bound."""
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


def applies(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, window: Grid) -> bool:
    """Whether `neighborhood_attention` computes this call (:160-167): the path switched on,
    matching fp16 CUDA tensors, and a shape and window `supports` admits."""
    if not _enabled or k.shape != q.shape or v.shape != q.shape:
        return False
    if any(t.dtype != torch.float16 or not t.is_cuda for t in (q, k, v)):
        return False
    return supports(tuple(int(size) for size in q.shape), window)


def neighborhood_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                           window: Grid) -> torch.Tensor:
    """Exact neighborhood attention of scaled (batch, T, H, W, heads, 64) fp16 queries over keys
    and values of the same shape with the inward-shifted `window` (:170-211); call it where
    `applies` holds. The output has the queries' shape and dtype."""
    if not applies(q, k, v, window=window):
        raise ValueError(f"neighborhood attention does not take {tuple(q.shape)} {q.dtype} "
                         f"arrays with window {window}")
    return ops.neighborhood_attention(q.contiguous(), k.contiguous(), v.contiguous(),
                                      window=tuple(window))


__all__ = ["HEAD_DIM", "applies", "enabled", "launch_fits", "neighborhood_attention",
           "run_tile", "set_enabled", "supports"]
