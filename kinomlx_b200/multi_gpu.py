"""Multi-GPU forms of the denoise step and the VAE decode that have an exchange step.

- CFG split: ranks [0, P/2) run the conditional branch and ranks [P/2, P)
  the unconditional one, each half with Ulysses sequence parallelism over its P/2 ranks. Rank r
  and rank r +- P/2 hold the same token shard; they all-gather their two velocity shards
  (kinomlx/models/flux2/sampling.py:264-280 combines the branches as `u + g * (p - u)`) and both
  apply the same Euler update.
- VAE tile scatter (config 5): the spatial tiles go round-robin to the ranks; each rank blends its
  tiles into a full-size fp32 canvas and the canvases and weight maps are summed before the
  normalisation (kinomlx/models/ltx2/video_vae/tiling.py:1310-1369): onto one owner rank (an
  NCCL reduce, half the bytes an all-reduce moves) when only that rank needs the video, or onto
  every rank (all-reduce).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .dist import shard_round_robin
from .sequence_parallel import SequenceParallel


class CfgSplit:
    """Process groups of the CFG split; every rank must construct it (same order of new_group)."""

    def __init__(self, *, peer: bool = False):
        """peer: Ulysses inside each branch over the peer transport instead of NCCL."""
        if not dist.is_initialized():
            raise RuntimeError("the CFG split needs an initialised process group")
        world, rank = dist.get_world_size(), dist.get_rank()
        if world % 2:
            raise ValueError("the CFG split needs an even number of ranks")
        half = world // 2
        branch_groups = [dist.new_group(list(range(half))), dist.new_group(list(range(half, world)))]
        pair_groups = [dist.new_group([i, i + half]) for i in range(half)]
        self.branch = 0 if rank < half else 1  # 0: conditional, 1: unconditional
        self.sp = SequenceParallel(branch_groups[self.branch], peer=peer)
        self.pair = pair_groups[rank % half]

    def combine(self, velocity: torch.Tensor, guidance: float) -> torch.Tensor:
        """Both branches' velocity shards -> u + g * (p - u) for this token shard."""
        both = [torch.empty_like(velocity) for _ in range(2)]
        dist.all_gather(both, velocity.contiguous(), group=self.pair)
        return ops.cfg_combine(both[0], both[1], guidance)


def cfg_split_step(model, prepared, current: torch.Tensor, sigmas: torch.Tensor, index: int,
                   guidance: float, cfg: CfgSplit) -> torch.Tensor:
    """One Klein Euler step of batched CFG with the two branches on different GPUs; `prepared`
    holds this rank's branch text (positive or negative) and `model.sp` is `cfg.sp`."""
    from .flux2.sampling import step_delta, timestep_x1000

    t = float(timestep_x1000(sigmas, index, 1))
    velocity = model.run(prepared, current, t)
    combined = cfg.combine(velocity, guidance)
    return ops.euler_velocity(current, combined, step_delta(sigmas, index), out=current)


def combine_canvases(canvas: torch.Tensor, weights: torch.Tensor, *, group=None,
                     dst: int | None = None) -> bool:
    """Sum every rank's blended canvas and weight map: onto rank `dst` of `group` (NCCL reduce),
    or, with `dst` None, onto every rank (all-reduce). Returns whether this rank holds the sums."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return True
    if dst is None:
        dist.all_reduce(canvas, group=group)
        dist.all_reduce(weights, group=group)
        return True
    root = dist.get_global_rank(group, dst) if group is not None else dst
    dist.reduce(canvas, root, group=group)
    dist.reduce(weights, root, group=group)
    return dist.get_rank(group) == dst


def decode_tiles_distributed(decoder, latent: torch.Tensor, *, tile: int = 8, overlap: int = 2,
                             group=None, dst: int | None = None) -> torch.Tensor | None:
    """Tiled VAE decode with the tiles spread round-robin over the ranks of `group`. With `dst`
    the decoded video is assembled on that rank only (the others return None); without it, on
    every rank."""
    from .ltx2.video_vae import tile_plan

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    _, _, f, h, w = latent.shape
    plan = tile_plan(h, w, tile, overlap, decoder.spatial_scale)
    mine = shard_round_robin(len(plan), world, rank)
    frames = f
    for blk in decoder.v.blocks:
        if blk[0] == "d2s" and blk[1][0] == 2:
            frames = 2 * frames - 1
    scale = decoder.spatial_scale
    canvas = torch.zeros((1, decoder.v.out_channels, frames, h * scale, w * scale),
                         device=decoder.device, dtype=torch.float32)
    weights = torch.zeros((h * scale, w * scale), device=decoder.device, dtype=torch.float32)
    if mine:
        decoder.decode_tiled(latent, tile=tile, overlap=overlap, tiles=mine,
                             canvas=canvas, weights=weights)
    if not combine_canvases(canvas, weights, group=group, dst=dst):
        return None
    return ops.blend_normalize(canvas, weights)
