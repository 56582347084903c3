"""One process per GPU: the host-side plumbing of the multi-GPU paths.

The reference has no distributed code; these helpers decide which work units a rank owns and
time collectives-free replicas. The data-path collectives (CFG velocity all-gather, Ulysses
all-to-all) go through torch.distributed on NCCL; the CPU tests run the same logic on gloo.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def world() -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment (1, 0, 0 without it)."""
    return (
        int(os.environ.get("WORLD_SIZE", "1")),
        int(os.environ.get("RANK", "0")),
        int(os.environ.get("LOCAL_RANK", "0")),
    )


def init(backend: str = "nccl", timeout_s: float = 120.0) -> None:
    """Join the process group with a short timeout, so ranks that wait on a missing peer end
    with an error instead of hanging."""
    size, rank, local = world()
    if size == 1 or dist.is_initialized():
        return
    kwargs = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)


def max_over_ranks(value: float) -> float:
    """The max of a host scalar over all ranks (step times are reported this way)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard_round_robin(units: int, size: int, rank: int) -> list[int]:
    """Units (e.g. the 15 VAE tiles of config 5) owned by `rank`: rank, rank + size, ..."""
    if size < 1 or not 0 <= rank < size:
        raise ValueError("rank must lie in [0, size)")
    return list(range(rank, units, size))


def token_shards(tokens: int, size: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) token ranges for sequence parallelism; the first ranks take the
    remainder so the ranges differ by at most one token."""
    base, extra = divmod(tokens, size)
    out, start = [], 0
    for r in range(size):
        end = start + base + (1 if r < extra else 0)
        out.append((start, end))
        start = end
    return out


def head_shards(heads: int, size: int) -> list[tuple[int, int]]:
    """Head ranges for the attention phase of Ulysses sequence parallelism; heads must divide."""
    if heads % size:
        raise ValueError(f"{heads} heads do not split over {size} ranks")
    per = heads // size
    return [(r * per, (r + 1) * per) for r in range(size)]


def cfg_groups(size: int) -> list[list[int]]:
    """CFG split: ranks [0, size/2) run the conditional branch, the rest the unconditional one;
    with size > 2 each half also shards tokens (Ulysses) inside its group."""
    if size == 1:
        return [[0]]
    if size % 2:
        raise ValueError("the CFG split needs an even number of ranks")
    half = size // 2
    return [list(range(half)), list(range(half, size))]
