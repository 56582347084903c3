"""Device twins of `kinomlx.samplers` (the Euler steps of kinomlx/samplers/steps.py)."""

from .steps import euler_step, euler_velocity_step

__all__ = ["euler_step", "euler_velocity_step"]
