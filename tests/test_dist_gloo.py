"""The multi-GPU host logic on two gloo ranks (CPU): work ownership, token/head shards and the
max-over-ranks timing reduction that bench.py uses."""

from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, size: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(size),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    from kinomlx_b200 import dist

    dist.init("gloo", timeout_s=30)
    owned = dist.shard_round_robin(15, size, rank)
    worst = dist.max_over_ranks(10.0 + rank)
    import torch.distributed as tdist

    gathered = [None] * size
    tdist.all_gather_object(gathered, owned)
    tdist.destroy_process_group()
    queue.put((rank, owned, worst, gathered))


def test_two_gloo_ranks_partition_and_reduce():
    size = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, size, port, queue)) for r in range(size)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(size)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, owned, worst, gathered in results:
        assert worst == 11.0
        flat = sorted(u for part in gathered for u in part)
        assert flat == list(range(15))  # every VAE tile exactly once
        assert owned == list(range(rank, 15, size))


def test_shard_helpers():
    from kinomlx_b200 import dist

    assert dist.token_shards(9216, 8) == [(i * 1152, (i + 1) * 1152) for i in range(8)]
    assert dist.token_shards(10, 4) == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert dist.head_shards(24, 8) == [(3 * i, 3 * i + 3) for i in range(8)]
    with pytest.raises(ValueError):
        dist.head_shards(24, 5)
    assert dist.cfg_groups(4) == [[0, 1], [2, 3]]
