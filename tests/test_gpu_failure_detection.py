"""Failure detection on the device without faulting it: a bounded wait that runs out.

The cross-GPU arrival barrier (kino_peer_barrier) is launched for rank 0 of a world of 2 on one
GPU, with both ranks' flag arrays in this GPU's memory and no rank 1 launched: the flag rank 0
waits for is never set. The wait gives up after its limit (2 s), records KINO_ETIMEOUT in the
device error word and returns; kino_device_status reports it on the host and clears it, and the
context stays usable. No kernel here faults, traps or waits without a limit, and only one
waiting kernel is ever launched."""

from __future__ import annotations

import pytest
import torch

from kinomlx_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _flags(world: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    flags = torch.zeros((world, world), dtype=torch.int32, device=device)
    ptrs = torch.tensor([flags[r].data_ptr() for r in range(world)], dtype=torch.int64,
                        device=device)
    return flags, ptrs


def test_barrier_wait_on_a_missing_rank_times_out(cuda_device):
    flags, ptrs = _flags(2, cuda_device)
    ops.peer_barrier(ptrs, 0, 2, 1)
    with pytest.raises(RuntimeError, match="timed out"):
        ops.device_status()
    # rank 0 published its arrival before waiting
    assert flags[0, 0].item() == 1 and flags[1, 0].item() == 1
    # the error word was cleared and the context still runs work
    ops.device_status()
    one, one_ptrs = _flags(1, cuda_device)
    ops.peer_barrier(one_ptrs, 0, 1, 1)  # a world of one passes at once
    ops.device_status()
    x = torch.randn((256, 64), device=cuda_device).to(torch.bfloat16)
    assert torch.equal(ops.gelu_tanh(x), ops.gelu_tanh(x))
    assert _lib.load().kino_device_status(None) == _lib.KINO_OK


def test_barrier_passes_when_every_arrival_is_present(cuda_device):
    """The same launch with rank 1's arrival already in place completes without an error."""
    flags, ptrs = _flags(2, cuda_device)
    flags[0, 1] = 1  # rank 1 arrived at barrier 1
    ops.peer_barrier(ptrs, 0, 2, 1)
    ops.device_status()
    assert flags[1, 0].item() == 1
