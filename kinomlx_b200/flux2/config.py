"""Shapes of the Flux2-style MMDiT: the reference's Klein graph and BASELINE's timed variant."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class FluxVariant:
    """What differs between the reference's Klein 9B graph
    (kinomlx/models/flux2/transformer.py:17-29, 63-65, 110-111, 185-186) and the timed configs."""

    dim: int
    heads: int
    mlp: str  # "gelu_tanh" or "swiglu"
    mlp_hidden: int  # activation width entering the MLP down projection
    rope_axes: tuple[int, ...]  # rotary dims per position axis (sum = head_dim)
    rope_theta: float
    in_channels: int
    context_dim: int
    double_blocks: int
    single_blocks: int
    head_dim: int = 128

    @property
    def mlp_in(self) -> int:
        return 2 * self.mlp_hidden if self.mlp == "swiglu" else self.mlp_hidden

    def with_blocks(self, double: int, single: int) -> "FluxVariant":
        return FluxVariant(
            self.dim, self.heads, self.mlp, self.mlp_hidden, self.rope_axes, self.rope_theta,
            self.in_channels, self.context_dim, double, single, self.head_dim,
        )


BASELINE = FluxVariant(
    dim=3072,
    heads=24,
    mlp="gelu_tanh",
    mlp_hidden=12288,
    rope_axes=(64, 64),
    rope_theta=10000.0,
    in_channels=64,
    context_dim=4096,
    double_blocks=8,
    single_blocks=24,
)

KLEIN = FluxVariant(
    dim=4096,
    heads=32,
    mlp="swiglu",
    mlp_hidden=12288,
    rope_axes=(32, 32, 32, 32),
    rope_theta=2000.0,
    in_channels=128,
    context_dim=12288,
    double_blocks=8,
    single_blocks=24,
)
