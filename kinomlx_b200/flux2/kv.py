"""Reference-token keys and values for Klein KV editing, owned by one denoising call
(kinomlx/models/flux2/kv.py:8-45).

The first evaluation of an edit runs [reference, target] image rows and stores, per layer, the
reference rows' keys (after QK RMSNorm and RoPE) and values; later evaluations run the target
rows only and attend to [own keys, stored reference keys] as two key segments of one attention
launch (softmax does not depend on key order). One allocation holds every layer:
(layers, 2, batch, reference tokens, width) in the model dtype, 2 * 32 * Nr * D * 2 bytes for
Klein at batch 1 (Nr = 4096: 2.1 GB).
"""

from __future__ import annotations

import torch


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
