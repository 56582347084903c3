"""Buffers shared over NVLink by the GPUs of a process group (one process per GPU, one node).

Each rank cudaMallocs its own buffer through the C ABI (kino_peer_alloc), the IPC handles are
exchanged with torch.distributed.all_gather_object, and every rank maps every other rank's buffer
(kino_peer_open). A shared buffer is then this rank's torch view plus an int64 device tensor of
all ranks' addresses, which kernels take as their `world`-entry pointer array. The arrival
barrier (kino_peer_barrier) runs on the stream between a kernel that writes into other GPUs'
buffers and the kernel that reads them.

No counterpart in the reference, which runs on one device.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import ops

_TYPESTR = {torch.bfloat16: "<i2", torch.int32: "<i4", torch.float32: "<f4"}


class _DeviceArray:
    """A raw device allocation exposed through __cuda_array_interface__ (no ownership)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3,
            "strides": None,
        }


def _view(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device):
    t = torch.as_tensor(_DeviceArray(ptr, shape, _TYPESTR[dtype]), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


class PeerGroup:
    """Shared buffers and a barrier over the ranks of `group` (collective calls throughout)."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 32:
            raise ValueError("peer groups span at most 32 GPUs")
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._owned: list[int] = []
        self._opened: list[int] = []
        self.epoch = 0
        _, self.flag_ptrs = self.shared((self.world,), torch.int32)

    def shared(self, shape: tuple[int, ...], dtype: torch.dtype = torch.bfloat16):
        """(this rank's zero-filled tensor of `shape`, int64 device tensor of all ranks' addresses)."""
        nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        ptr, handle = ops.peer_alloc(max(256, nbytes))
        self._owned.append(ptr)
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(ptr)
            else:
                peer = ops.peer_open(h)
                self._opened.append(peer)
                ptrs.append(peer)
        local = _view(ptr, shape, dtype, self.device)
        return local, torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def barrier(self) -> None:
        """Every rank's earlier kernels' stores are visible to all ranks after this point on the
        stream (device-side; bounded wait)."""
        self.epoch += 1
        ops.peer_barrier(self.flag_ptrs, self.rank, self.world, self.epoch)

    def close(self) -> None:
        """Unmap and free, after every rank has finished with every buffer."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            ops.peer_close(p)
        self._opened.clear()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._owned:
            ops.peer_free(p)
        self._owned.clear()
