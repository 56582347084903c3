"""Flux2-style MMDiT denoise step on the B200 kernels."""
