"""Token positions of a patch-size-1 video latent grid (kinomlx/models/ltx2/patchifier.py:102-146,
kinomlx/models/ltx2/conditioning/tools.py:63-74): the (1, 3, tokens, 2) pixel-space [start, end)
bounds of each latent voxel in row-major (frame, row, column) order, the time axis shifted by the
causal fix (first frame covers one pixel frame) and divided by the frame rate. Host arithmetic,
computed once per generation; the RoPE tables are built from it."""

from __future__ import annotations

import torch


def latent_positions(frames: int, height: int, width: int, *, scale=(8, 32, 32),
                     causal_fix: bool = True, fps: float = 24.0) -> torch.Tensor:
    f, h, w = torch.meshgrid(torch.arange(frames), torch.arange(height), torch.arange(width),
                             indexing="ij")
    starts = torch.stack([f, h, w]).reshape(3, -1).to(torch.float32)
    bounds = torch.stack([starts, starts + 1], dim=-1)[None]
    pix = bounds * torch.tensor(scale, dtype=torch.float32).reshape(1, 3, 1, 1)
    if causal_fix:
        pix[:, 0] = torch.clamp(pix[:, 0] + 1 - scale[0], min=0)
    pix[:, 0] = pix[:, 0] / fps
    return pix
