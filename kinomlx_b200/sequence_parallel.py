"""Ulysses sequence parallelism around attention (one process per GPU, NCCL all-to-all).

The reference runs on one device; this is the multi-GPU form of its attention calls. Each rank
holds a contiguous share of the tokens for every projection, norm and MLP. Around each
self-attention, q, k and v go through one all-to-all each (token shards -> head shards: every rank
then sees all tokens for heads/P heads), the attention kernel runs on that block, and one
all-to-all brings the output back to token shards. Softmax attention does not depend on the order
of its keys, so the rank-major token order of the gathered sequence is exact.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


class SequenceParallel:
    """All-to-all attention over the ranks of `group` (None: the default group)."""

    def __init__(self, group=None, *, local: bool = False):
        self.group = group
        initialised = dist.is_available() and dist.is_initialized() and not local
        self.size = dist.get_world_size(group) if initialised else 1
        self.rank = dist.get_rank(group) if initialised else 0
        self._buffers: dict[tuple, tuple] = {}

    @classmethod
    def single(cls) -> "SequenceParallel":
        """No sharding: every token on this GPU (the default of the models)."""
        return cls(local=True)

    def shard(self, length: int) -> tuple[int, int]:
        """This rank's [start, end) of a length divisible by the group size."""
        if length % self.size:
            raise ValueError(f"{length} tokens do not split evenly over {self.size} ranks")
        per = length // self.size
        return self.rank * per, (self.rank + 1) * per

    def _bufs(self, tokens: int, width: int, device) -> tuple:
        key = (tokens, width, device)
        if key not in self._buffers:
            p = self.size
            mk = lambda: torch.empty((p, tokens, width // p), device=device, dtype=torch.bfloat16)
            self._buffers[key] = tuple(mk() for _ in range(8))
        return self._buffers[key]

    def attention(self, q, k, v, out, *, heads: int, gate=None) -> None:
        """q, k, v, out: (1, local tokens, heads * 128) views; gate: (1, local tokens, heads)."""
        if self.size == 1:
            ops.attention([q], [k], [v], [out], heads=heads, gate=None if gate is None else [gate])
            return
        p = self.size
        if heads % p:
            raise ValueError(f"{heads} heads do not split over {p} ranks")
        tokens, width = q.shape[1], q.shape[2]
        sq, sk, sv, rq, rk, rv, att, ro = self._bufs(tokens, width, q.device)
        for src, send, recv in ((q, sq, rq), (k, sk, rk), (v, sv, rv)):
            ops.heads_pack(src[0], p, out=send)
            dist.all_to_all_single(recv, send, group=self.group)
        full = lambda t: t.view(1, p * tokens, width // p)
        ops.attention([full(rq)], [full(rk)], [full(rv)], [full(att)], heads=heads // p)
        dist.all_to_all_single(ro, att, group=self.group)
        ops.heads_unpack(ro, out[0], gate=None if gate is None else gate[0])

    def all_gather_tokens(self, local: torch.Tensor) -> torch.Tensor:
        """(1, tokens/P, C) shards -> (1, tokens, C) in rank order."""
        if self.size == 1:
            return local
        parts = [torch.empty_like(local) for _ in range(self.size)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)
