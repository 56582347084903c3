"""Shape of the LTX-2 video stream (kinomlx/models/ltx2/transformer/model.py:137-170)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class LTXVariant:
    dim: int = 4096
    heads: int = 32
    head_dim: int = 128
    context_dim: int = 4096
    ff_mult: int = 4
    gated_attention: bool = True
    eps: float = 1e-6
    theta: float = 10000.0
    max_pos: tuple[int, int, int] = (20, 2048, 2048)
    in_channels: int = 128
    out_channels: int = 128
    blocks: int = 48
    timestep_scale: float = 1000.0

    def with_blocks(self, blocks: int) -> "LTXVariant":
        return LTXVariant(self.dim, self.heads, self.head_dim, self.context_dim, self.ff_mult,
                          self.gated_attention, self.eps, self.theta, self.max_pos,
                          self.in_channels, self.out_channels, blocks, self.timestep_scale)


# hidden 4096, 32 x 128 heads, 48 blocks, 256 text tokens of width 4096.
BASELINE_VIDEO = LTXVariant()
