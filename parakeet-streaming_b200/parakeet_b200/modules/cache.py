"""Paged streaming cache: the drop-in for ``ModelCache``/``StreamingState``
(parakeet/modules/cache.py:7-95).

``PagedModelCache`` is the batch view of a ``PagedKVPool`` for the slots of
one step.  It keeps the reference's method names and return shapes:

* ``update_attn_cache(layer, key, value)`` appends the chunk's rows into the
  stream's pages and returns the dense [B, left+T, D] windows, bit-identical
  to the reference's shifted window (cache.py:36-45);
* ``get_conv_cache(layer)`` returns a handle that the paged
  ``ConformerConvolution`` updates in place; ``update_conv_cache`` accepts it
  (or a dense [B, D, K-1] tensor) like cache.py:47-53.

The attention and conv modules of this package read the pages and the conv
cache in place through ``pool`` and ``slots`` instead of the dense copies.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..ops import PagedKVPool


class ConvCacheRef:
    """The conv time cache of one layer for the batch's slots, by reference."""

    def __init__(self, cache: "PagedModelCache", layer_idx: int):
        self.cache = cache
        self.layer_idx = layer_idx

    def tensor(self) -> torch.Tensor:
        """Dense copy [B, D, K-1] (reference layout)."""
        return self.cache.pool.conv[self.cache.slots.long(), self.layer_idx]

    def size(self, dim=None):
        shape = (self.cache.batch_size, self.cache.pool.dim, self.cache.conv_cache_len)
        return torch.Size(shape) if dim is None else shape[dim]


class PagedModelCache:
    def __init__(self, pool: PagedKVPool, slots: torch.Tensor, lengths: torch.Tensor | None = None):
        self.pool = pool
        self.slots = slots                      # int32 [B] on the pool's device
        self.lengths = lengths                  # int32 [B], set per step by the encoder
        self.left_attn = pool.left
        self.right_attn = pool.chunk - 1
        self.attn_context_size = (self.left_attn, self.right_attn)
        self.attn_cache_len = pool.window
        self.conv_cache_len = pool.conv_kernel - 1

    @property
    def batch_size(self) -> int:
        return int(self.slots.numel())

    def update_attn_cache(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor):
        self.pool.append(layer_idx, key, value, self.slots)
        return self.pool.gather(layer_idx, self.slots)

    def get_conv_cache(self, layer_idx: int) -> ConvCacheRef:
        return ConvCacheRef(self, layer_idx)

    def update_conv_cache(self, layer_idx: int, state) -> None:
        if state is None or isinstance(state, ConvCacheRef):
            return                               # already updated in place
        self.pool.conv[self.slots.long(), layer_idx] = state.to(self.pool.dtype)

    def reset_slot(self, slot: int) -> None:
        """Zero the conv cache of a pool slot; its pages are returned by the
        scheduler's release path."""
        self.pool.zero_conv_slot(int(self.slots[slot]))


@dataclass
class StreamingState:
    """``StreamingState`` (cache.py:80-89) over a paged cache; the counters
    are read from the pool's per-slot metadata."""

    cache: PagedModelCache

    @property
    def processed_frames(self) -> torch.Tensor:
        return self.cache.pool.counters(self.cache.slots)[0]

    @property
    def cache_lengths(self) -> torch.Tensor:
        return self.cache.pool.counters(self.cache.slots)[1]

    def attn_cache_len(self) -> int:
        return int(self.cache_lengths.max().item()) if self.cache.batch_size else 0


ModelCache = PagedModelCache

__all__ = ["PagedModelCache", "ModelCache", "ConvCacheRef", "StreamingState"]
