"""kino_group_norm_noalloc: GroupNorm(32) + SiLU for callers that cannot allocate device memory.

Some hosts own every device allocation themselves (a plugin living inside a media or inference
server with a fixed memory budget) or must not call cudaMalloc/cudaFree while a pipeline runs,
because those calls can synchronise the device. They cannot hand kino_group_norm the workspace
its cross-block statistics need, so this entry point keeps that scratch in a fixed array inside
the library. This test calls it through the C ABI and checks it against kino_group_norm with a
caller workspace: both launch the same kernels with the same partition count, so the outputs
must be bit-identical. Three calls in a row, small, large, then small again with other
statistics, so a call that read past its own partitions or kept a previous call's scratch would
see the larger call's leftovers.

Kept in a file of its own that pytest collects last, so a failure here comes after every other
test has run; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

BF = torch.bfloat16


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def test_group_norm_noalloc_matches_workspace_entry_point(cuda_device):
    from kinomlx_b200 import _lib

    lib = _lib.load()
    header = (Path(__file__).resolve().parents[1] / "include" / "kino.h").read_text()
    limit = int(re.search(r"#define KINO_GROUP_NORM_NOALLOC_SCRATCH_BYTES (\d+)", header).group(1))
    # every accepted shape fits the static scratch (the partition count is capped)
    assert lib.kino_group_norm_workspace_size(1 << 40, 2048) <= limit

    gen = torch.Generator().manual_seed(2024)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = (((1, 4, 33, 8, 512), 0, 1.0), ((1, 9, 17, 23, 256), 1, 2.0),
             ((1, 4, 33, 8, 512), 1, 5.0))
    for shape, silu, scale in cases:
        c = shape[-1]
        voxels = 1
        for s in shape[:-1]:
            voxels *= s
        x = (torch.randn(shape, generator=gen) * scale + scale).to(BF).to(cuda_device)
        w = (torch.randn(c, generator=gen) * 0.5 + 1.0).to(BF).to(cuda_device)
        b = (torch.randn(c, generator=gen) * 0.1).to(BF).to(cuda_device)
        expect = torch.empty_like(x)
        out = torch.full_like(x, float("nan"))
        need = int(lib.kino_group_norm_workspace_size(voxels, c))
        workspace = torch.empty(need, dtype=torch.uint8, device=cuda_device)
        status = lib.kino_group_norm(_p(x), _p(w), _p(b), _p(expect), voxels, c, 1e-6, silu,
                                     _p(workspace), need, stream)
        assert status == 0, _lib.last_error()
        status = lib.kino_group_norm_noalloc(_p(x), _p(w), _p(b), _p(out), voxels, c, 1e-6, silu,
                                             stream)
        assert status == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert bool(torch.isfinite(out).all())
        assert torch.equal(out, expect), float((out.float() - expect.float()).abs().max())
