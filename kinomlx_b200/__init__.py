"""kinomlx_b200: the denoise-step hot path of KinoMLX on B200 (sm_100a).

The compute lives in libkino_b200.so (hand-written tcgen05/TMA kernels behind the C ABI of
include/kino.h). This package holds the host side: the ctypes binding (_lib), torch-tensor
wrappers (ops), the reference-shaped op surface (kernels) and the model call sites that drive
one denoise step (flux2, ltx2, samplers).
"""

__version__ = "0.1.0"
