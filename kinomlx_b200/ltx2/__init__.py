"""LTX-2 video DiT (video stream) on the B200 kernels."""
