"""Build libkino_b200.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/kino_capi.cu includes every kernel header), linked
against the static CUDA runtime; the TMA descriptor encoder is reached through
cudaGetDriverEntryPoint, so no libcuda link is needed at build time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "libkino_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "kino.h"]


def needs_build() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(path.stat().st_mtime > built for path in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/kino_capi.cu into libkino_b200.so next to this file."""
    if not force and not needs_build():
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        *ARCH_FLAGS,
        *NVCC_FLAGS,
        f"-I{INCLUDE}",
        str(CSRC / "kino_capi.cu"),
        "-o",
        str(tmp),
    ]
    result = subprocess.run(cmd, capture_output=True, text=True)
    log = result.stdout + result.stderr
    (PACKAGE / "build.log").write_text(log)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{log[-6000:]}")
    if verbose:
        print(log)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
