"""Features -> tokens for a batch of streams in one call: the batched
counterpart of the reference engine's per-chunk work (``_run_pre_encode``,
``_encode_step``, ``_decode_batch``; parakeet/engine/model_runner.py:181-447).

One ``step`` runs the batched pre-encode (per-slot mel cache), the paged
streaming encoder (per-slot K/V pages and conv cache) and the batched greedy
decode (per-slot prediction state) for the same slots, with no host read-back
in between, so a steady-state step can be captured in one CUDA graph.  Every
per-stream state is indexed by the stream's slot, as the reference's encoder
state is (parakeet/engine/scheduler.py:86-104).
"""
from __future__ import annotations

import torch

from ..modules.cache import PagedModelCache, StreamingState
from .decoding import BatchedGreedyDecoder
from .pre_encode import BatchedPreEncoder


class StreamingPipeline:
    def __init__(self, encoder, pre_encode, predictor, joiner, blank_id: int, num_slots: int,
                 max_symbols: int = 5, **pool_kw):
        p = next(encoder.parameters())
        self.device, self.dtype = p.device, p.dtype
        self.encoder = encoder
        self.pool = encoder.make_pool(num_slots, device=self.device, dtype=self.dtype, **pool_kw)
        self.pre = BatchedPreEncoder(pre_encode, num_slots,
                                     cache_size=encoder.pre_encode_cache_size[1],
                                     drop_extra=encoder.drop_extra_pre_encoded)
        self.dec = BatchedGreedyDecoder(predictor, joiner, blank_id, num_slots, max_symbols)

    def start_streams(self, slots) -> None:
        """Fresh state for new streams in ``slots`` (their pages start empty;
        conv cache and prediction state as ``create_sequence`` leaves them)."""
        for s in torch.as_tensor(slots).reshape(-1).tolist():
            self.pool.zero_conv_slot(int(s))
        self.dec.reset_slots(slots)

    def end_streams(self, slots) -> None:
        """Finished streams: their pages return to the pool at the next step."""
        for s in torch.as_tensor(slots).reshape(-1).tolist():
            self.pool.release_slot(int(s))

    def step(self, feats: torch.Tensor, slots: torch.Tensor, first: bool):
        """feats [B, feat_in, frames] of one chunk per stream (all first
        chunks, or all later chunks), slots int32 [B] on the device.  Returns
        tokens int32 [B, T, max_symbols] (-1 = none) and counts int32 [B, T]."""
        x = self.pre.pre_encode(feats, slots, first)                 # [B, T, D]
        state = StreamingState(PagedModelCache(self.pool, slots))
        y, _ = self.encoder(x, state, bypass_pre_encode=True)        # [B, D, T]
        B, T = x.shape[:2]
        lengths = torch.full((B,), T, dtype=torch.int32, device=self.device)
        return self.dec.decode(y.transpose(1, 2), lengths, slots)


__all__ = ["StreamingPipeline"]
