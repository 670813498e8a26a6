"""Audio -> tokens for a batch of streams in one call: the batched
counterpart of the reference engine's per-chunk work (``_run_pre_encode``
with its ``FeatureExtractor.push``, ``_encode_step``, ``_decode_batch``;
parakeet/engine/model_runner.py:181-447).

``step_audio`` runs the batched log-mel extractor (per-slot sample history),
then ``step``: the batched pre-encode (per-slot mel cache), the paged
streaming encoder (per-slot K/V pages and conv cache) and the batched greedy
decode (per-slot prediction state), for the same slots, with no host
read-back in between, so a steady-state step can be captured in one CUDA
graph.  Every per-stream state is indexed by the stream's slot, as the
reference's encoder state is (parakeet/engine/scheduler.py:86-104).

Chunking follows the reference engine (model_runner.py:53-56,94-95): a
stream's first chunk has (1 + 8 * lookahead) hops of samples and emits
8 * lookahead mel frames (the last hop's window is not complete yet), later
chunks (8 + 8 * lookahead) hops and as many frames.  The pre-encode cache
keeps the last 9 frames of each window, or a whole first window shorter than
that (8 frames for lookahead 1), so a stream's second window is shorter than
the later ones; after the subsampling ((F - 2) // 8 + 2 frames of F) and the
2-frame drop of cached windows every push gives exactly lookahead + 1
encoder frames, one encoder chunk.  Rows of one batch are at the same push
index (first, second, later), because their windows have the same length.
"""
from __future__ import annotations

import torch

from .. import _lib
from ..modules.cache import PagedModelCache, StreamingState
from ..modules.features import FeatureExtractor, frames_emitted
from .decoding import BatchedGreedyDecoder
from .pre_encode import BatchedPreEncoder


class StreamingPipeline:
    def __init__(self, encoder, pre_encode, predictor, joiner, blank_id: int, num_slots: int,
                 max_symbols: int = 5, feature_kw: dict | None = None, **pool_kw):
        """``feature_kw``: FeatureExtractor arguments (the reference's defaults
        otherwise, dither included); n_mels is the pre-encoder's feat_in."""
        p = next(encoder.parameters())
        self.device, self.dtype = p.device, p.dtype
        self.encoder = encoder
        self.pool = encoder.make_pool(num_slots, device=self.device, dtype=self.dtype, **pool_kw)
        self.pre = BatchedPreEncoder(pre_encode, num_slots,
                                     cache_size=encoder.pre_encode_cache_size[1],
                                     drop_extra=encoder.drop_extra_pre_encoded)
        self.dec = BatchedGreedyDecoder(predictor, joiner, blank_id, num_slots, max_symbols)
        self.fe = FeatureExtractor(**{"n_mels": self.pre.feat_in, **(feature_kw or {})},
                                   num_slots=num_slots, device=self.device, out_dtype=self.dtype)
        self._fe_bufs = {}

    def start_streams(self, slots) -> None:
        """Fresh state for new streams in ``slots`` (their pages start empty;
        conv cache and prediction state as ``create_sequence`` leaves them; the
        feature history restarts with their first ``step_audio``)."""
        for s in torch.as_tensor(slots).reshape(-1).tolist():
            self.pool.zero_conv_slot(int(s))
        self.dec.reset_slots(slots)
        self.fe.reset_slots(slots)

    def frames_per_push(self, n: int, first: bool) -> int:
        """Mel frames a push of ``n`` samples emits: on a first push the
        reference rule; on later pushes of whole hops exactly n / hop (the
        window end advances by n samples, first pushes longer than n_fft / 2)."""
        hop, n_fft = self.fe.hop_length, self.fe.n_fft
        if first:
            return frames_emitted(0, 0, n, False, hop, n_fft)
        if n % hop:
            raise ValueError(f"later chunks are whole hops of {hop} samples, got {n}")
        return n // hop

    def step_audio(self, samples: torch.Tensor, slots: torch.Tensor, push: int,
                   first_samples: int | None = None):
        """samples float32 [B, n] on the device: one chunk of audio per stream,
        every stream at push index ``push`` (0 = its first chunk); slots int32
        [B] on the device.  ``first_samples``: the size of the streams' first
        chunk (needed at push 1 to know how many frames the pre-encode cache
        holds; default the engine's first chunk, (1 + 8 * lookahead) hops).
        Returns tokens int32 [B, T, max_symbols] (-1 = none) and counts int32
        [B, T]."""
        B, n = samples.shape
        first = push == 0
        F = self.frames_per_push(n, first)
        prefix = None
        if push == 1:
            if first_samples is None:
                la = self.encoder.att_context_size[1]
                first_samples = (1 + 8 * la) * self.fe.hop_length
            prefix = min(self.frames_per_push(first_samples, True), self.pre.cache_size)
        key = (B, n, first)
        bufs = self._fe_bufs.get(key)
        if bufs is None:
            dev = self.device
            bufs = (torch.full((B,), n, dtype=torch.int32, device=dev),
                    torch.full((B,), _lib.PK_FE_FIRST if first else 0, dtype=torch.int32,
                               device=dev),
                    torch.empty(B, self.fe.n_mels, F, dtype=self.dtype, device=dev),
                    torch.empty(B, dtype=torch.int32, device=dev))
            self._fe_bufs[key] = bufs
        ns, flags, feats, nframes = bufs
        self.fe.launch(samples, ns, flags, slots, feats, F, nframes)
        return self.step(feats, slots, first, prefix=prefix)

    def end_streams(self, slots) -> None:
        """Finished streams: their pages return to the pool at the next step."""
        for s in torch.as_tensor(slots).reshape(-1).tolist():
            self.pool.release_slot(int(s))

    def step(self, feats: torch.Tensor, slots: torch.Tensor, first: bool,
             prefix: int | None = None):
        """feats [B, feat_in, frames] of one chunk per stream (all first
        chunks, or all later chunks), slots int32 [B] on the device; ``prefix``
        the cached feature frames to prepend (BatchedPreEncoder.pre_encode).
        Returns tokens int32 [B, T, max_symbols] (-1 = none) and counts int32
        [B, T]."""
        x = self.pre.pre_encode(feats, slots, first, prefix)         # [B, T, D]
        state = StreamingState(PagedModelCache(self.pool, slots))
        y, _ = self.encoder(x, state, bypass_pre_encode=True)        # [B, D, T]
        B, T = x.shape[:2]
        lengths = torch.full((B,), T, dtype=torch.int32, device=self.device)
        return self.dec.decode(y.transpose(1, 2), lengths, slots)


__all__ = ["StreamingPipeline"]
