"""Batched streaming pre-encode: the convolutional subsampling of many streams'
feature chunks in one call, with every stream's mel-frame cache in a device
pool indexed by its encoder slot.

The reference runs ``_run_pre_encode`` (parakeet/engine/model_runner.py:
181-233) once per stream per chunk: it concatenates the stream's cached
feature frames and the new chunk, runs ``ConvSubsampling`` on a batch of one,
drops ``drop_extra_pre_encoded`` leading output frames when a cache was used,
and keeps the last ``pre_encode_cache_size`` input frames as the next cache.
Here ``pk_pre_encode_window`` builds the cache-prefixed inputs of a whole batch
and advances all their caches in one launch, and the subsampling runs once on
the batch.  A stream's first chunk (no cache yet) has a different length from
the following ones, so callers batch first chunks and later chunks separately.
"""
from __future__ import annotations

import torch

from .._lib import check, lib
from ..ops import DTYPES, _stream


class BatchedPreEncoder:
    def __init__(self, pre_encode, num_slots: int, cache_size: int = 9, drop_extra: int = 2):
        p = next(pre_encode.parameters())
        self.device, self.dtype = p.device, p.dtype
        if self.dtype not in DTYPES:
            raise ValueError(f"dtype {self.dtype} not handled")
        self.module, self.feat_in = pre_encode, pre_encode.feat_in
        self.cache_size, self.drop_extra, self.num_slots = cache_size, drop_extra, num_slots
        self.cache = torch.zeros(num_slots, self.feat_in, cache_size, dtype=self.dtype,
                                 device=self.device)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)

    def pre_encode(self, feats: torch.Tensor, slots: torch.Tensor, first: bool,
                   prefix: int | None = None) -> torch.Tensor:
        """feats [B, feat_in, frames] (the feature extractor's layout), slots
        [B]; ``first``: the streams' first chunks (no cache); ``prefix``: the
        cached frames to prepend (default: the cache size; fewer after a first
        chunk shorter than the cache, which the cache then holds whole,
        model_runner.py:225-230).  Returns the pre-encoded frames [B, frames',
        hidden] and advances the caches."""
        B, M, F = feats.shape
        if M != self.feat_in:
            raise ValueError(f"{M} feature bins, the subsampling takes {self.feat_in}")
        pre = 0 if first else (self.cache_size if prefix is None else int(prefix))
        if not 0 <= pre <= self.cache_size:
            raise ValueError(f"prefix {pre} outside [0, {self.cache_size}]")
        feats = feats.to(device=self.device, dtype=self.dtype).contiguous()
        sl = slots.to(device=self.device, dtype=torch.int32).contiguous()
        x = torch.empty(B, M, pre + F, dtype=self.dtype, device=self.device)
        check(lib().pk_pre_encode_window(self.cache.data_ptr(), self.num_slots, feats.data_ptr(),
                                         sl.data_ptr(), B, M, F, self.cache_size, pre,
                                         x.data_ptr(), DTYPES[self.dtype], self.error.data_ptr(),
                                         _stream(self.device)), "pk_pre_encode_window")
        drop = 0 if first else self.drop_extra
        if self.module.stream_supported(x):
            return self.module.forward_stream(x, drop)      # fused convs, dropped rows skipped
        y = self.module.forward_full(x.transpose(1, 2))   # every row spans all frames
        return y[:, drop:] if drop else y


__all__ = ["BatchedPreEncoder"]
