"""Reference-token keys and values for Klein KV editing, owned by one denoising call
(kinomlx/models/flux2/kv.py:8-45).

The first evaluation of an edit runs [reference, target] image rows and stores, per layer, the
reference rows' keys (after QK RMSNorm and RoPE) and values; later evaluations run the target
rows only and attend to [own keys, stored reference keys] as two key segments of one attention
launch (softmax does not depend on key order). One allocation holds every layer:
(layers, 2, batch, reference tokens, width) in the model dtype, 2 * 32 * Nr * D * 2 bytes for
Klein at batch 1 (Nr = 4096: 2.1 GB). `attend_rows` is the attention the transformer runs on
its projection rows; `reference_attention` is the reference's function on (batch, tokens, heads,
d) tensors.
"""

from __future__ import annotations

import torch

from .. import ops


class ReferenceKV:
    def __init__(self, reference_tokens: int, layers: int, batch: int, width: int,
                 device: torch.device, dtype: torch.dtype):
        if reference_tokens < 1 or layers < 1:
            raise ValueError("Reference K/V requires positive token and layer counts")
        self.reference_tokens = reference_tokens
        self.layer_count = layers
        self.batch = batch
        self._store: torch.Tensor | None = torch.empty(
            (layers, 2, batch, reference_tokens, width), device=device, dtype=dtype)
        self._filled = [False] * layers
        self.extracting = True
        self.closed = False

    def keep(self, layer: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Copy one layer's reference rows (batch, Nr, width) into the store."""
        if self._store is None:
            raise ValueError("Reference K/V belongs to a completed generation")
        self._store[layer, 0].copy_(key)
        self._store[layer, 1].copy_(value)
        self._filled[layer] = True

    def tensors(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self._store is None or not self._filled[layer]:
            raise ValueError("Reference K/V has not been extracted")
        return self._store[layer, 0], self._store[layer, 1]

    def clear(self) -> None:
        """Release the store; the cache cannot be used again."""
        self._store = None
        self._filled = [False] * self.layer_count
        self.closed = True


def attend_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, heads: int,
                text_tokens: int, state: ReferenceKV, layer: int) -> None:
    """Attention with reference K/V on post-RoPE (batch, rows, heads * d) bf16 rows, written to
    `out` (which may be q): reusing, rows are [text, target] and the kept reference rows join as
    a second key segment; extracting, rows are [text, reference, target], the reference rows'
    keys/values are kept, text and target queries attend to every key and reference queries to
    the reference keys only (kinomlx/models/flux2/kv.py:57-80)."""
    if not state.extracting:
        rk, rv = state.tensors(layer)
        ops.attention([q], [k, rk], [v, rv], [out], heads=heads)
        return
    r0, r1 = text_tokens, text_tokens + state.reference_tokens
    state.keep(layer, k[:, r0:r1], v[:, r0:r1])
    active = [(a, b) for a, b in ((0, r0), (r1, q.shape[1])) if b > a]
    if active:
        ops.attention([q[:, a:b] for a, b in active], [k], [v], [out[:, a:b] for a, b in active],
                      heads=heads)
    ops.attention([q[:, r0:r1]], [k[:, r0:r1]], [v[:, r0:r1]], [out[:, r0:r1]], heads=heads)


def reference_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, *,
                        text_tokens: int, state: ReferenceKV, layer: int) -> torch.Tensor:
    """The reference's function (kinomlx/models/flux2/kv.py:57-80) on post-RoPE
    (batch, tokens, heads, d) bf16 device tensors, d 64 or 128; returns the same shape."""
    b, n, h, d = query.shape
    if key.shape != query.shape or value.shape != query.shape:
        raise ValueError("query, key and value must share one (batch, tokens, heads, d) shape")
    q, k, v = (x.reshape(b, n, h * d) for x in (query, key, value))
    out = torch.empty_like(q)
    attend_rows(q, k, v, out, heads=h, text_tokens=text_tokens, state=state, layer=layer)
    return out.reshape(b, n, h, d)
