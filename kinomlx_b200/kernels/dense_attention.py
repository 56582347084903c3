"""`kinomlx.models.ltx2.kernels.dense_attention` surface
(kinomlx/models/ltx2/kernels/dense_attention.py:87-151) on the tcgen05 attention kernel.

bf16 in and out with fp32 softmax and accumulation (no fp16 saturation: the reference converts
only because the M1 lacks bf16 arithmetic). Heads are 64 or 128 wide, as the reference's kernel
takes (dense_attention.py:87-104).
"""

from __future__ import annotations

import torch

from .. import ops

HEAD_DIMS = (64, 128)
_SUPPORTED = (torch.bfloat16,)


def applies(query: torch.Tensor, key: torch.Tensor, *, heads: int) -> bool:
    return (
        query.dim() == 3
        and key.dim() == 3
        and query.dtype in _SUPPORTED
        and key.dtype == query.dtype
        and query.shape[0] == key.shape[0]
        and query.shape[-1] == key.shape[-1]
        and query.shape[-1] in tuple(heads * d for d in HEAD_DIMS)
        and query.shape[1] > 0
        and key.shape[1] > 0
        and query.is_cuda
    )


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int) -> torch.Tensor:
    """Dense attention of (query_tokens, heads*dim) queries over (key_tokens, heads*dim) keys."""
    if q.dtype not in _SUPPORTED or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"dense attention needs bfloat16 q, k and v, got {q.dtype}, {k.dtype}, {v.dtype}")
    width = q.shape[1] if q.dim() == 2 else 0
    dim = width // heads if heads > 0 and width % heads == 0 else 0
    if dim not in HEAD_DIMS or k.dim() != 2 or k.shape[1] != width or v.shape != k.shape or q.shape[0] == 0 or k.shape[0] == 0:
        raise ValueError(
            f"dense attention needs (query_tokens, {heads} * 64 or 128) queries and matching "
            f"(key_tokens, width) keys and values, got {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}"
        )
    out = torch.empty_like(q)
    ops.attention([q[None]], [k[None]], [v[None]], [out[None]], heads=heads)
    return out
