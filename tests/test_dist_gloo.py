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


class _CpuOps:
    """CPU stand-ins for the three device ops SequenceParallel launches, so its all-to-all
    ordering and layout logic can run on gloo ranks."""

    @staticmethod
    def heads_pack(src, parts, out):
        tokens, width = src.shape
        out.copy_(src.reshape(tokens, parts, width // parts).transpose(0, 1))
        return out

    @staticmethod
    def heads_unpack(src, out, gate=None):
        parts, tokens, chunk = src.shape
        rows = src.transpose(0, 1).reshape(tokens, parts * chunk)
        if gate is not None:
            rows = (rows.reshape(tokens, -1, 128) * gate[..., None]).reshape(tokens, -1)
        out.copy_(rows)
        return out

    @staticmethod
    def attention(q, k, v, out, heads, gate=None, kv_splits=1):
        from oracle.fused_ops import sdpa

        b, t, w = q[0].shape
        d = w // heads
        split = lambda x: x.reshape(b, x.shape[1], heads, d).transpose(1, 2)
        o = sdpa(split(q[0]), split(k[0]), split(v[0]), d ** -0.5).transpose(1, 2).reshape(b, t, w)
        out[0].copy_(o)


def _sp_worker(rank: int, size: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(size),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import torch

    from kinomlx_b200 import dist, sequence_parallel

    sequence_parallel.ops = _CpuOps
    dist.init("gloo", timeout_s=60)
    heads, tokens = 4, 12
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((1, tokens, heads * 128), generator=gen).to(torch.bfloat16) for _ in range(3))
    gate = torch.rand((1, tokens, heads), generator=gen).to(torch.bfloat16)
    sp = sequence_parallel.SequenceParallel()
    t0, t1 = sp.shard(tokens)
    out = torch.zeros((1, t1 - t0, heads * 128), dtype=torch.bfloat16)
    sp.attention(q[:, t0:t1], k[:, t0:t1], v[:, t0:t1], out, heads=heads, gate=gate[:, t0:t1])
    full = sp.all_gather_tokens(out)
    import torch.distributed as tdist

    tdist.destroy_process_group()
    queue.put((rank, full.float().numpy().tolist()))


def test_two_gloo_ranks_ulysses_attention_equals_full_attention():
    """The sequence-parallel all-to-all attention on 2 gloo ranks equals one-device attention
    with the per-head gate (the layout and ordering logic that runs on NCCL on the GPUs)."""
    import torch

    from oracle.fused_ops import sdpa

    size, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_sp_worker, args=(r, size, port, queue)) for r in range(size)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=180) for _ in range(size))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    heads, tokens = 4, 12
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((1, tokens, heads * 128), generator=gen).to(torch.bfloat16) for _ in range(3))
    gate = torch.rand((1, tokens, heads), generator=gen).to(torch.bfloat16)
    split = lambda x: x.reshape(1, tokens, heads, 128).transpose(1, 2)
    o = sdpa(split(q), split(k), split(v), 128 ** -0.5).transpose(1, 2)
    expect = (o * gate[..., None]).reshape(1, tokens, heads * 128)
    for r in range(size):
        assert torch.equal(torch.tensor(results[r]).to(torch.bfloat16), expect)


def _qkv(branch: int, heads: int, tokens: int):
    import torch

    gen = torch.Generator().manual_seed(40 + branch)
    return tuple(torch.randn((1, tokens, heads * 128), generator=gen).to(torch.bfloat16)
                 for _ in range(3))


def _cfg_worker(rank: int, size: int, port: int, queue) -> None:
    """One rank of the CFG split: the branch's Ulysses attention over its half of the ranks,
    then the pair combine u + g (p - u) of the two branches' shards."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(size),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as tdist

    from kinomlx_b200 import dist, multi_gpu, sequence_parallel

    sequence_parallel.ops = _CpuOps
    multi_gpu.ops = type("CpuCfg", (), {
        "cfg_combine": staticmethod(lambda p, u, g: (u.float() + g * (p.float() - u.float())).to(p.dtype))})
    dist.init("gloo", timeout_s=60)
    cfg = multi_gpu.CfgSplit()
    heads, tokens = 4, 8
    q, k, v = _qkv(cfg.branch, heads, tokens)
    t0, t1 = cfg.sp.shard(tokens)
    out = torch.zeros((1, t1 - t0, heads * 128), dtype=torch.bfloat16)
    cfg.sp.attention(q[:, t0:t1], k[:, t0:t1], v[:, t0:t1], out, heads=heads)
    combined = cfg.combine(out, 3.0)
    full = cfg.sp.all_gather_tokens(combined)
    pair = tdist.get_process_group_ranks(cfg.pair)
    tdist.destroy_process_group()
    queue.put((rank, cfg.branch, cfg.sp.size, pair, full.float().numpy().tolist()))


@pytest.mark.parametrize("size", [2, 4])
def test_gloo_ranks_cfg_split_with_ulysses_branches(size):
    """CFG split on 2 ranks (one branch each) and 4 ranks (each branch on a Ulysses group of 2,
    BASELINE config 3's layout at 4 GPUs): every rank ends with u + g (p - u) of the whole
    sequence, p and u the two branches' full attention outputs."""
    import torch

    from oracle.fused_ops import sdpa

    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_cfg_worker, args=(r, size, port, queue)) for r in range(size)]
    for p in procs:
        p.start()
    results = {r: rest for r, *rest in (queue.get(timeout=240) for _ in range(size))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    heads, tokens, half = 4, 8, size // 2
    outs = []
    for branch in (0, 1):
        q, k, v = _qkv(branch, heads, tokens)
        split = lambda x: x.reshape(1, tokens, heads, 128).transpose(1, 2)
        o = sdpa(split(q), split(k), split(v), 128 ** -0.5).transpose(1, 2).reshape(1, tokens, -1)
        outs.append(o.to(torch.bfloat16))
    expect = (outs[1].float() + 3.0 * (outs[0].float() - outs[1].float())).to(torch.bfloat16)
    for rank, (branch, sp_size, pair, full) in results.items():
        assert branch == (0 if rank < half else 1) and sp_size == half
        assert pair == [rank % half, rank % half + half]
        assert torch.equal(torch.tensor(full).to(torch.bfloat16), expect)


def _canvas_worker(rank: int, size: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(size),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import torch

    from kinomlx_b200 import dist
    from kinomlx_b200.multi_gpu import combine_canvases

    dist.init("gloo", timeout_s=30)
    out = {}
    for dst in (None, 1):
        canvas = torch.full((1, 3, 2, 4, 5), float(rank + 1))
        weights = torch.full((4, 5), 0.5 * (rank + 1))
        holds = combine_canvases(canvas, weights, dst=dst)
        out[dst] = (holds, float(canvas.max()) if holds else None, float(weights.max()) if holds else None)
    import torch.distributed as tdist

    tdist.destroy_process_group()
    queue.put((rank, out))


def test_gloo_ranks_combine_tile_canvases():
    """The VAE tile canvases: summed onto every rank (all-reduce) or onto one owner rank
    (reduce), which alone reports that it holds the sums."""
    size = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_canvas_worker, args=(r, size, port, queue)) for r in range(size)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(size))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(size):
        assert results[rank][None] == (True, 3.0, 1.5)
    assert results[1][1] == (True, 3.0, 1.5)
    assert results[0][1] == (False, None, None)
