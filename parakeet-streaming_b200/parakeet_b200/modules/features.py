"""Streaming log-mel feature extraction on the GPU, batched over streams.

``FeatureExtractor`` is a drop-in for the reference's extractor
(parakeet/modules/feature_extractor.py:8-151): same constructor arguments and
attributes, same ``__call__(audio)`` and ``push(samples, state, final)``
results.  The reference keeps each stream's recent samples in a host buffer
and recomputes an STFT over it at every push; here every stream slot keeps
its last ``PK_FE_HIST`` samples and its counters on the device and one
``pk_features_push`` launch computes only the new frames, for any number of
streams at once (``push_batch``).

A stream's slot is its encoder slot (``state.encoder_state`` in ``push``,
like the reference's scheduler pool, parakeet/engine/scheduler.py:86-104).
The device counters are authoritative; a host mirror of them (samples seen,
frames emitted per slot) only sizes the outputs, because a push's frame
count depends on sample counts alone.

Dither: the reference adds ``torch.randn`` noise of std ``dither`` to the
retained samples at every push.  Here the noise of a sample comes from a
counter-based generator (Philox-4x32-10) keyed by (seed, slot, stream, sample
index): the same distribution, reproducible for a given seed.  Outputs are
on the extractor's device (the reference returns CPU tensors).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from .. import _lib
from .._lib import check, lib
from ..ops import DTYPES, _stream


def frames_emitted(total_before: int, emitted_before: int, n: int, final: bool, hop: int,
                   n_fft: int) -> int:
    """Frames a push of ``n`` samples emits (feature_extractor.py:97-125)."""
    if n == 0:
        return 0
    total = total_before + n
    if final:
        last = total // hop
    elif total <= n_fft // 2:
        return 0
    else:
        last = (total - n_fft // 2) // hop
    return max(0, last - emitted_before + 1)


class FeatureExtractor:
    model_input_names = ["input_features"]

    def __init__(self, sampling_rate=16000, n_mels=128, n_fft=512, window_size=0.025,
                 window_stride=0.01, normalize="NA", preemph=0.97, dither=1e-5,
                 log_zero_guard_value=2 ** -24, lowfreq=0, highfreq=None, mag_power=2.0,
                 pad_value=0.0, mel_norm="slaney", *, num_slots: int = 1, device=None,
                 out_dtype=torch.float32, seed: int = 0):
        self.sampling_rate = sampling_rate
        self.feature_size = n_mels
        self.padding_value = pad_value
        self.normalize = normalize
        self.n_mels = n_mels
        self.n_fft = n_fft or 2 ** math.ceil(math.log2(int(window_size * sampling_rate)))
        self.win_length = int(window_size * sampling_rate)
        self.hop_length = int(window_stride * sampling_rate)
        self.preemph = preemph
        self.dither = dither
        self.log_zero_guard_value = float(log_zero_guard_value)
        self.mag_power = mag_power
        self.pad_value = pad_value
        self.window = torch.hann_window(self.win_length, periodic=False)
        highfreq = highfreq or sampling_rate / 2
        norm = {"slaney": 1, None: 0}.get(mel_norm)
        if norm is None:
            raise ValueError(f"mel_norm {mel_norm!r}: 'slaney' or None")
        if out_dtype not in DTYPES:
            raise ValueError(f"out_dtype {out_dtype} not handled")
        self.device = torch.device(device if device is not None else "cuda")
        self.out_dtype = out_dtype

        nbytes, nnz = ctypes.c_int64(), ctypes.c_int32()
        args = (sampling_rate, self.n_fft, self.win_length, n_mels, float(lowfreq),
                float(highfreq), norm)
        check(lib().pk_features_tables(*args, None, ctypes.byref(nbytes), ctypes.byref(nnz)),
              "pk_features_tables")
        host = np.zeros(nbytes.value // 4, np.int32)
        check(lib().pk_features_tables(*args, host.ctypes.data, ctypes.byref(nbytes),
                                       ctypes.byref(nnz)), "pk_features_tables")
        self.mel_nnz = nnz.value
        self.fb = self._dense_filters(host)                 # [n_mels, n_fft // 2 + 1], host
        self.tables = torch.from_numpy(host).to(self.device)

        # one extra slot serves __call__ (whole utterances)
        self.num_slots = num_slots
        self._call_slot = num_slots
        S = num_slots + 1
        self.history = torch.zeros(S, _lib.PK_FE_HIST, dtype=torch.float32, device=self.device)
        self.meta = torch.zeros(S, _lib.PK_FE_META_STRIDE, dtype=torch.int64, device=self.device)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._seen = np.zeros(S, np.int64)
        self._emitted = np.zeros(S, np.int64)
        self.desc = _lib.FeaturesDesc(
            tables=self.tables.data_ptr(), history=self.history.data_ptr(),
            meta=self.meta.data_ptr(), error=self.error.data_ptr(), num_slots=S,
            n_fft=self.n_fft, hop=self.hop_length, n_mels=n_mels, mel_nnz=self.mel_nnz,
            preemph=preemph, dither=dither, mag_power=mag_power,
            log_guard=self.log_zero_guard_value, pad_value=pad_value,
            seed=seed & 0xFFFFFFFFFFFFFFFF)

    def _dense_filters(self, words: np.ndarray) -> torch.Tensor:
        n_fft, n_mels, nnz = self.n_fft, self.n_mels, self.mel_nnz
        base = 16 + 3 * n_fft
        lo, cnt, off = (words[base + i * n_mels:base + (i + 1) * n_mels] for i in range(3))
        w = words[base + 3 * n_mels:base + 3 * n_mels + nnz].view(np.float32)
        fb = np.zeros((n_mels, n_fft // 2 + 1), np.float32)
        for m in range(n_mels):
            fb[m, lo[m]:lo[m] + cnt[m]] = w[off[m]:off[m] + cnt[m]]
        return torch.from_numpy(fb)

    # ------------------------------------------------------------ batched
    def frames_for(self, slot: int, n: int, first: bool, final: bool) -> int:
        seen = 0 if first else int(self._seen[slot])
        emitted = 0 if first else int(self._emitted[slot])
        return frames_emitted(seen, emitted, n, final, self.hop_length, self.n_fft)

    def launch(self, samples: torch.Tensor, num_samples: torch.Tensor, flags: torch.Tensor,
               slots: torch.Tensor, out: torch.Tensor | None, max_frames: int,
               num_frames: torch.Tensor) -> None:
        """Raw device push (graph-capturable, leaves the host mirror alone):
        samples float32 [B, ld] and int32 [B] num_samples / flags / slots /
        num_frames, all on the device; out [B, n_mels, max_frames]."""
        if self.device.type != "cuda":
            raise RuntimeError("pk_features_push runs on a CUDA device; this extractor's "
                               f"state lives on {self.device}")
        B = samples.shape[0]
        if out is not None and (out.dtype != self.out_dtype or not out.is_contiguous()
                                or tuple(out.shape) != (B, self.n_mels, max_frames)):
            raise ValueError("out must be a contiguous [B, n_mels, max_frames] tensor of out_dtype")
        if samples.dtype != torch.float32 or samples.stride(-1) != 1:
            raise ValueError("samples must be float32 rows with unit stride")
        check(lib().pk_features_push(
            ctypes.byref(self.desc), samples.data_ptr() or None,
            samples.stride(0) if B and samples.shape[1] else 0,
            num_samples.data_ptr(), flags.data_ptr(), slots.data_ptr(), B,
            out.data_ptr() if out is not None else None, DTYPES[self.out_dtype], max_frames,
            num_frames.data_ptr(), _stream(self.device)), "pk_features_push")

    def push_batch(self, samples, slots, first=False, final=False, num_samples=None,
                   out: torch.Tensor | None = None):
        """One push for a batch of streams.  samples float32 [B, n] (host or
        device), slots host ints [B]; ``first`` / ``final`` a bool or one per
        row; ``num_samples`` per-row counts <= n (default n).  Returns
        (features [B, n_mels, F] with F the largest frame count, pad_value past
        a row's count; frame counts np.int64 [B])."""
        slots_np = np.asarray(torch.as_tensor(slots).cpu(), np.int64).reshape(-1)
        B = slots_np.size
        if B and (slots_np.min() < 0 or slots_np.max() >= self.num_slots + 1):
            raise ValueError("slot outside the pool")
        if np.unique(slots_np).size != B:
            raise ValueError("a slot appears twice in one push")
        x = torch.as_tensor(samples, dtype=torch.float32)
        if x.dim() == 1:
            x = x.reshape(1, -1)
        if x.shape[0] != B:
            raise ValueError(f"{x.shape[0]} sample rows for {B} slots")
        n = np.full(B, x.shape[1], np.int64) if num_samples is None else \
            np.asarray(num_samples, np.int64).reshape(-1)
        if n.size != B or (B and (n.min() < 0 or n.max() > x.shape[1])):
            raise ValueError("num_samples outside [0, samples per row]")
        first = np.broadcast_to(np.asarray(first, bool), (B,))
        final = np.broadcast_to(np.asarray(final, bool), (B,))
        counts = np.array([self.frames_for(int(s), int(k), bool(a), bool(b))
                           for s, k, a, b in zip(slots_np, n, first, final)], np.int64)
        F = int(counts.max()) if B else 0
        flags = first.astype(np.int32) * _lib.PK_FE_FIRST + final.astype(np.int32) * _lib.PK_FE_FINAL
        dev = self.device
        meta = torch.from_numpy(np.stack([n.astype(np.int32), flags.astype(np.int32),
                                          slots_np.astype(np.int32)])).to(dev, non_blocking=True)
        x = x.to(dev, non_blocking=True).contiguous()
        if out is None:
            out = torch.empty(B, self.n_mels, F, dtype=self.out_dtype, device=dev)
        nframes = torch.empty(B, dtype=torch.int32, device=dev)
        self.launch(x, meta[0], meta[1], meta[2], out if F else None, F, nframes)
        for s, k, a, c in zip(slots_np, n, first, counts):
            if a:
                self._seen[s], self._emitted[s] = 0, 0
            self._seen[s] += k
            self._emitted[s] += c
        return out, counts

    def reset_slots(self, slots) -> None:
        """Forget the host mirror of ``slots``; their next push must be first."""
        for s in np.asarray(torch.as_tensor(slots).cpu(), np.int64).reshape(-1):
            self._seen[s] = self._emitted[s] = 0

    # ------------------------------------------------------------ reference API
    def __call__(self, audio, return_tensors: str | None = None, padding: bool = True):
        """Log-mel features [1, n_mels, 1 + len(audio) // hop] of a whole
        utterance (``FeatureExtractor.__call__``, feature_extractor.py:90-95)."""
        assert isinstance(audio, np.ndarray)
        assert audio.ndim == 1
        if audio.size == 0:
            raise ValueError("empty audio")
        out, _ = self.push_batch(audio.reshape(1, -1), [self._call_slot], first=True, final=True)
        return out

    def push(self, samples: np.ndarray, state, final: bool = False):
        """``FeatureExtractor.push`` (feature_extractor.py:97-133): the new
        frames [1, n_mels, F] of the stream whose slot is ``state.encoder_state``,
        or None.  The state's ``_fe_emitted_frames`` / ``_fe_sample_offset``
        keep the frames emitted and the samples consumed (the samples
        themselves stay on the device), so a state the reference would treat
        as fresh (both 0 and no retained samples) starts a new stream."""
        if not samples.size:
            return None
        slot = int(state.encoder_state)
        first = (state._fe_emitted_frames == 0 and state._fe_sample_offset == 0
                 and getattr(state, "_fe_samples", np.empty(0)).size == 0)
        out, counts = self.push_batch(samples.reshape(1, -1), [slot], first=first, final=final)
        state._fe_emitted_frames = int(self._emitted[slot])
        state._fe_sample_offset = int(self._seen[slot])
        return out if counts[0] > 0 else None

    def error_bits(self) -> int:
        return int(self.error.item())


__all__ = ["FeatureExtractor", "frames_emitted"]
