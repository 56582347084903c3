"""Sol-Attn routed sparse attention restated on the CPU (test oracle; nothing else may import it).

Follows kinomlx/models/ltx2/kernels/sol_attention.py:1-275 and its Metal bodies
(kinomlx/models/ltx2/kernels/metal/sol_attention_prepare.metal:1-53,
sol_attention_body.metal:1-378), which implement the published Sol-Attn of NVlabs' Sana
Sol-Engine (Apache-2.0): tokens in 64-token blocks along a 3-D Morton curve; each query block
scores every key block by mean query against mean key and routes the blocks above
mean + tau * std of those scores (diagonal key covariance), plus itself and both neighbours;
routed blocks are attended exactly, every other block through its mean key (score + log2 of the
block's length) and its mean value, all in one softmax.

Precision as the reference's kernel: q, k and v are gathered into routing order and converted to
fp16 with saturation at its largest finite value; the query means stay fp32 and the key and value
means are rounded to the input dtype, then to fp16; the scores and the softmax run in fp32.
Pinned in tests/test_sol_attention_oracle.py against the reference's own tests
(tests/models/ltx2/test_sol_attention.py).
"""

from __future__ import annotations

import math

import torch

BLOCK = 64
HEAD_DIM = 128
LOG2E = 1.4426950408889634
VARIANCE_EPSILON = 1.0e-6
FP16_MAX = 65504.0


def block_count(tokens: int) -> int:
    return (tokens + BLOCK - 1) // BLOCK


def morton_order(frames: int, height: int, width: int, *, tokens: int | None = None) -> torch.Tensor:
    """Raster indices of an (F, H, W) grid listed along a 3-D Morton curve: bit i of the frame,
    row and column index goes to bits 3i, 3i + 1 and 3i + 2 of a token's code; tokens past the
    grid keep their order after it (sol_attention.py:106-136)."""
    if min(frames, height, width) <= 0:
        raise ValueError("Morton order needs positive grid dimensions")
    grid = frames * height * width
    total = grid if tokens is None else tokens
    if total < grid:
        raise ValueError(f"{total} tokens cannot hold a {frames}x{height}x{width} grid")
    bits = max(frames, height, width).bit_length()

    def interleaved(size: int, shift: int) -> torch.Tensor:
        idx = torch.arange(size, dtype=torch.int64)
        code = torch.zeros_like(idx)
        for bit in range(bits):
            code |= ((idx >> bit) & 1) << (3 * bit + shift)
        return code

    codes = (interleaved(frames, 0)[:, None, None] | interleaved(height, 1)[None, :, None]
             | interleaved(width, 2)[None, None, :]).reshape(-1)
    order = torch.argsort(codes, stable=True)
    if total > grid:
        order = torch.cat([order, torch.arange(grid, total)])
    return order


def _to_fp16(x: torch.Tensor) -> torch.Tensor:
    """The kernel dtype conversion: saturate at fp16's largest finite value (exact inside its
    normal range)."""
    return x.float().clamp(-FP16_MAX, FP16_MAX).half()


def prepare(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, order: torch.Tensor):
    """Gather into routing order and take the 64-token block means: fp16 q, k, v (tokens, H*D),
    fp32 query means and fp16 key/value means rounded through the input dtype, each
    (heads, blocks, D) (sol_attention_prepare.metal:11-53)."""
    tokens = q.shape[0]
    blocks = block_count(tokens)
    gathered = [x[order] for x in (q, k, v)]
    pad = blocks * BLOCK - tokens
    lengths = torch.clamp(tokens - torch.arange(blocks) * BLOCK, max=BLOCK).float()

    def means(x: torch.Tensor) -> torch.Tensor:
        f = torch.nn.functional.pad(x.float(), (0, 0, 0, pad))
        sums = f.reshape(blocks, BLOCK, heads, HEAD_DIM).sum(dim=1)
        return (sums / lengths[:, None, None]).transpose(0, 1).contiguous()

    qmean = means(gathered[0])
    kmean = _to_fp16(means(gathered[1]).to(q.dtype))
    vmean = _to_fp16(means(gathered[2]).to(q.dtype))
    return (*(_to_fp16(x) for x in gathered), qmean, kmean, vmean)


def route_blocks(qmean: torch.Tensor, kmean: torch.Tensor, *, tau: float):
    """Routing from block means (sol_attention.py:181-216): key block b is routed for query block
    a when |a - b| <= 1 or its log2-scaled score exceeds the row's mean + tau * std under a
    diagonal key covariance. Returns the (H, NB, NB) routes, each row's ascending routed blocks
    followed by the rest, the counts and the 32-bit mask words."""
    heads, blocks, dim = qmean.shape
    keys = kmean.float()
    log2_scale = dim ** -0.5 * LOG2E
    scores = (qmean @ keys.transpose(1, 2)) * log2_scale
    center = keys.mean(dim=1, keepdim=True)
    raw_mean = (qmean * center).sum(-1)
    key_variance = ((keys - center) ** 2).mean(dim=1, keepdim=True)
    raw_variance = (qmean ** 2 * key_variance).sum(-1)
    variance = torch.clamp(raw_variance, min=0.0) * (log2_scale * log2_scale)
    limit = raw_mean * log2_scale + tau * torch.sqrt(variance + VARIANCE_EPSILON)
    index = torch.arange(blocks)
    neighbour = (index[:, None] - index[None, :]).abs() <= 1
    routes = neighbour[None] | (scores > limit[..., None])
    counts = routes.sum(-1).to(torch.int32)
    lists = torch.argsort(torch.where(routes, index, index + blocks), dim=-1, stable=True)
    words = (blocks + 31) // 32
    padded = torch.nn.functional.pad(routes, (0, words * 32 - blocks)).to(torch.int64)
    weights = torch.tensor([1 << i for i in range(32)], dtype=torch.int64)
    bits = (padded.reshape(heads, blocks, words, 32) * weights).sum(-1)
    return routes, lists, counts, bits


def attend(q16, k16, v16, kmean, vmean, routes) -> torch.Tensor:
    """The attention in routing order (sol_attention_body.metal:7-14, 229-373): per query, the
    exact scores of the keys in its block's routed blocks and, for every other block, the score
    of its mean key plus log2 of the block's length with the block's mean value, in one base-2
    softmax; fp32 arithmetic on the fp16 operands. Returns (tokens, heads * D) fp32."""
    tokens = q16.shape[0]
    heads, blocks, dim = kmean.shape
    scale2 = LOG2E / math.sqrt(dim)
    token_block = torch.arange(tokens) // BLOCK
    lengths = torch.clamp(tokens - torch.arange(blocks) * BLOCK, max=BLOCK).float()
    out = []
    for h in range(heads):
        cols = slice(h * dim, (h + 1) * dim)
        qh, kh, vh = (x[:, cols].float() for x in (q16, k16, v16))
        routed = routes[h][token_block]  # (tokens, blocks): the query's block row
        exact = (qh @ kh.T) * scale2
        exact = exact.masked_fill(~routed[:, token_block], -math.inf)
        cent = (qh @ kmean[h].float().T) * scale2 + torch.log2(lengths)
        cent = cent.masked_fill(routed, -math.inf)
        peak = torch.maximum(exact.max(-1).values, cent.max(-1).values)[:, None]
        pe, pc = torch.exp2(exact - peak), torch.exp2(cent - peak)
        num = pe @ vh + pc @ vmean[h].float()
        out.append(num / (pe.sum(-1) + pc.sum(-1))[:, None])
    return torch.cat(out, dim=-1)


def sol_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, heads: int, tau: float,
                  order: torch.Tensor) -> torch.Tensor:
    """Sol-Attn of (tokens, heads * 128) fp16/bf16 inputs routed in `order`; the output comes
    back in the inputs' order and dtype (sol_attention.py:219-272)."""
    if not math.isfinite(tau):
        raise ValueError(f"Sol attention tau must be finite, got {tau}")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("Sol attention needs float16 or bfloat16 q, k and v")
    if q.dim() != 2 or q.shape[1] != heads * HEAD_DIM or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"Sol attention needs (tokens, {heads} * {HEAD_DIM}) q, k and v")
    if order.shape != (q.shape[0],):
        raise ValueError("the token order must hold one index per token")
    q16, k16, v16, qmean, kmean, vmean = prepare(q, k, v, heads=heads, order=order)
    routes, _, _, _ = route_blocks(qmean, kmean, tau=tau)
    routed_order = attend(q16, k16, v16, kmean, vmean, routes)
    out = torch.empty_like(routed_order)
    out[order] = routed_order
    return out.to(q.dtype)
