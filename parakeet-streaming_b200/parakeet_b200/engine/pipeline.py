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
        self._fe_bufs = {}          # recent batch sizes' feature buffers (bounded)
        self._fe_bufs_graph = {}    # buffers a captured CUDA graph uses: kept for good

    def start_streams(self, slots) -> None:
        """Fresh state for new streams in ``slots`` (their pages start empty;
        conv cache and prediction state as ``create_sequence`` leaves them; the
        feature history restarts with their first ``step_audio``)."""
        idx = torch.as_tensor(slots, dtype=torch.int64).reshape(-1).to(self.device)
        self.pool.conv.index_fill_(0, idx, 0)
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
        y, lengths = self.encode_audio(samples, slots, push, first_samples)
        return self.dec.decode(y, lengths, slots)

    def encode_audio(self, samples: torch.Tensor, slots: torch.Tensor, push: int,
                     first_samples: int | None = None):
        """The features, pre-encode and encoder half of ``step_audio``:
        returns the encoder output [B, T, D] and the frame counts int32 [B]."""
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
        capturing = torch.cuda.is_current_stream_capturing()
        bufs = self._fe_bufs_graph.get(key)
        if bufs is None:
            bufs = self._fe_bufs.pop(key, None)
        if bufs is None:
            while len(self._fe_bufs) >= 16:   # batches of many sizes: keep the recent ones
                self._fe_bufs.pop(next(iter(self._fe_bufs)))
            dev = self.device
            bufs = (torch.full((B,), n, dtype=torch.int32, device=dev),
                    torch.full((B,), _lib.PK_FE_FIRST if first else 0, dtype=torch.int32,
                               device=dev),
                    torch.empty(B, self.fe.n_mels, F, dtype=self.dtype, device=dev),
                    torch.empty(B, dtype=torch.int32, device=dev))
        ns, flags, feats, nframes = bufs
        if capturing or key in self._fe_bufs_graph:
            # a graph captured now reads these addresses at every replay: they
            # must outlive any eviction of the recent-sizes cache.  Graphs of
            # different push indices share them (same batch, samples and
            # first flag), so each graph, and each eager step on them, sets the
            # two constants itself: the fill that made them may sit in another
            # graph that has not been replayed yet.
            self._fe_bufs_graph[key] = bufs
            ns.fill_(n)
            flags.fill_(_lib.PK_FE_FIRST if first else 0)
        else:
            self._fe_bufs[key] = bufs
        self.fe.launch(samples, ns, flags, slots, feats, F, nframes)
        return self.encode(feats, slots, first, prefix=prefix)

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
        y, lengths = self.encode(feats, slots, first, prefix)
        return self.dec.decode(y, lengths, slots)

    def encode(self, feats: torch.Tensor, slots: torch.Tensor, first: bool,
               prefix: int | None = None):
        """Pre-encode and encoder half of ``step``: the encoder output [B, T, D]
        and the frame counts int32 [B]."""
        x = self.pre.pre_encode(feats, slots, first, prefix)         # [B, T, D]
        state = StreamingState(PagedModelCache(self.pool, slots))
        y, _ = self.encoder(x, state, bypass_pre_encode=True)        # [B, D, T]
        B, T = x.shape[:2]
        lengths = torch.full((B,), T, dtype=torch.int32, device=self.device)
        return y.transpose(1, 2), lengths


class OverlappedStreamingRunner:
    """Steady-state audio steps (push index 2 on) of one batch of streams, with
    chunk k's greedy decode on a second stream running under chunk k+1's
    features, pre-encode and encoder - the reference engine's separate encode
    and decode loops (parakeet/engine/model_runner.py:150-171) as two streams
    of CUDA graphs.  Two sets of graphs and buffers alternate (step k uses set
    k % 2); step k's encoder graph waits for step k-2's decode, the only one
    that read that set's encoder output.  Call after the pipeline has run at
    least one steady step eagerly for this batch (the capture needs its
    workspaces); ``slots`` and the batch stay fixed."""

    def __init__(self, pipe: StreamingPipeline, slots: torch.Tensor, samples_per_chunk: int):
        dev = pipe.device
        B = int(slots.numel())
        self.pipe, self.slots, self.device = pipe, slots, dev
        self.audio = [torch.zeros(B, samples_per_chunk, dtype=torch.float32, device=dev)
                      for _ in range(2)]
        self.dec_stream = torch.cuda.Stream(dev)
        self.enc_done = [torch.cuda.Event() for _ in range(2)]
        self.dec_done = [torch.cuda.Event() for _ in range(2)]
        self.g_enc, self.g_dec, self.out, self._y = [], [], [], []
        self.k = 0
        # The two sides are captured on different streams: library handles
        # that keep a workspace per stream (cuBLAS) then bake different
        # workspaces into the encoder and the decode graphs, which run at once.
        cap_e, cap_d = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        for cap in (cap_e, cap_d):
            cap.wait_stream(torch.cuda.current_stream(dev))
        for j in range(2):
            ge, gd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(ge, stream=cap_e):
                y, lengths = pipe.encode_audio(self.audio[j], slots, 2)
            cap_d.wait_stream(cap_e)
            with torch.cuda.graph(gd, stream=cap_d):
                tokens, counts = pipe.dec.decode(y, lengths, slots)
            self.g_enc.append(ge)
            self.g_dec.append(gd)
            self._y.append((y, lengths))
            self.out.append((tokens, counts))
        for cap in (cap_e, cap_d):
            torch.cuda.current_stream(dev).wait_stream(cap)

    def step(self, samples: torch.Tensor | None = None):
        """One steady step: copies ``samples`` (float32 [B, n], host or device)
        into this step's input set, launches its encoder side on the current
        stream and its decode on the decode stream.  Returns (tokens, counts,
        event): the tensors are final once ``event`` has completed and stay so
        until the call after next."""
        j = self.k % 2
        main = torch.cuda.current_stream(self.device)
        if self.k >= 2:
            main.wait_event(self.dec_done[j])
        if samples is not None:
            self.audio[j].copy_(samples, non_blocking=True)
        self.g_enc[j].replay()
        self.enc_done[j].record(main)
        self.dec_stream.wait_event(self.enc_done[j])
        with torch.cuda.stream(self.dec_stream):
            self.g_dec[j].replay()
        self.dec_done[j].record(self.dec_stream)
        self.k += 1
        tokens, counts = self.out[j]
        return tokens, counts, self.dec_done[j]

    def drain(self) -> None:
        """Make the current stream wait for every launched decode."""
        main = torch.cuda.current_stream(self.device)
        for e in self.dec_done:
            main.wait_event(e)


__all__ = ["StreamingPipeline", "OverlappedStreamingRunner"]
