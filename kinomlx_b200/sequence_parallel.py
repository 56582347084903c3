"""Ulysses sequence parallelism around attention (one process per GPU).

The reference runs on one device; this is the multi-GPU form of its attention calls. Each rank
holds a contiguous share of the tokens for every projection, norm and MLP; around each
self-attention, q, k and v move from token shards to head shards (every rank then sees all
tokens for heads/P heads), the attention kernel runs on that block, and the output moves back to
token shards. Softmax attention does not depend on the order of its keys, so the rank-major
token order of the gathered sequence is exact.

Two transports:
  peer (default on GPUs): the q/k/v projection's epilogue stores each head group's columns
      straight into the owning GPU's receive buffer over NVLink (ops.Scatter), a device-side
      arrival barrier follows, the attention stores each output row straight back into the
      token owner's projection buffer (ops.PeerReturn), and a second barrier closes the
      exchange. No separate copy, pack or collective kernel.
  nccl: pack -> all_to_all_single -> attention -> all_to_all_single -> unpack (gloo on CPU in the
      tests; the reference point for the peer transport).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


class SequenceParallel:
    """All-to-all attention over the ranks of `group` (None: the default group)."""

    def __init__(self, group=None, *, local: bool = False, peer: bool = False):
        self.group = group
        initialised = dist.is_available() and dist.is_initialized() and not local
        self.size = dist.get_world_size(group) if initialised else 1
        self.rank = dist.get_rank(group) if initialised else 0
        self._buffers: dict[tuple, tuple] = {}
        self.peer = None
        if peer and self.size > 1:
            from .peer import PeerGroup

            self.peer = PeerGroup(group)
        self._recv: dict[tuple, tuple] = {}

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
        ops.attention([full(rq)], [full(rk)], [full(rv)], [full(att)], heads=heads // p,
                      kv_splits="auto")
        dist.all_to_all_single(ro, att, group=self.group)
        ops.heads_unpack(ro, out[0], gate=None if gate is None else gate[0])

    # ------------------------------------------------------------------ peer transport
    def shared(self, shape: tuple[int, ...], dtype: torch.dtype = torch.bfloat16):
        """A buffer the other ranks can write into: (local tensor, device array of addresses)."""
        if self.peer is None:
            raise RuntimeError("shared buffers need the peer transport")
        return self.peer.shared(shape, dtype)

    def receive(self, local_tokens: int, width: int):
        """This rank's q/k/v receive buffer for `local_tokens` per rank and a model width:
        (P * local_tokens, 3 * width / P), slots [q | k | v], rows in rank-major token order."""
        key = (local_tokens, width)
        if key not in self._recv:
            self._recv[key] = self.shared((self.size * local_tokens, 3 * (width // self.size)))
        return self._recv[key]

    def scatter(self, recv_entry, width: int, slots: tuple[int, ...], local_row0: int) -> ops.Scatter:
        """Epilogue scatter of a projection whose first len(slots) column segments of `width` are
        q/k/v (slots[s] = 0, 1, 2 for q, k, v); its output row i is this rank's local token
        local_row0 + i."""
        recv, ptrs = recv_entry
        local_tokens = recv.shape[0] // self.size
        return ops.Scatter(ptrs, self.size, width, len(slots), recv.shape[1], recv.shape[0],
                           self.rank * local_tokens + local_row0, slots)

    def attention_from_peers(self, recv_entry, *, heads: int, out_ptrs: torch.Tensor,
                             out_ld: int, out_cols: int, out_col: int, gate=None) -> None:
        """Barrier, attention over this rank's head group of the gathered sequence with every
        row returned to its owner's output (columns out_col + this rank's head group), barrier.
        gate: (device array of the owners' gate buffers, their row stride) or None."""
        recv, _ = recv_entry
        p = self.size
        rows, w3 = recv.shape
        w = w3 // 3
        self.peer.barrier()
        q = recv[:, :w].unsqueeze(0)
        k = recv[:, w : 2 * w].unsqueeze(0)
        v = recv[:, 2 * w :].unsqueeze(0)
        ret = ops.PeerReturn(out_ptrs, p, rows // p, out_ld, out_cols, out_col + self.rank * w,
                             gate_ptrs=None if gate is None else gate[0],
                             ld_gate=0 if gate is None else gate[1],
                             gate_head_offset=self.rank * (heads // p))
        # H / P heads of the whole sequence: few query tiles, so the keys are split among CTAs
        # where that finishes sooner (ops.attention_splits)
        ops.attention([q], [k], [v], [q], heads=heads // p, peer_return=ret, kv_splits="auto")
        self.peer.barrier()

    def close(self) -> None:
        if self.peer is not None:
            self._recv.clear()
            self.peer.close()
            self.peer = None

    def all_gather_tokens(self, local: torch.Tensor) -> torch.Tensor:
        """(1, tokens/P, C) shards -> (1, tokens, C) in rank order."""
        if self.size == 1:
            return local
        parts = [torch.empty_like(local) for _ in range(self.size)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)
