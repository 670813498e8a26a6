"""float64 numpy restatement of the reference's streaming log-mel extractor.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Restates
``FeatureExtractor`` (parakeet/modules/feature_extractor.py):

* the constructor's derived constants (:28-57): win_length = 0.025 s and
  hop = 0.01 s in samples, a symmetric Hann window (``torch.hann_window(
  win_length, periodic=False)``), and the mel bank of
  ``librosa.filters.mel(norm="slaney")``.  librosa (``librosa>=0.11.0`` in the
  reference's pyproject.toml) is not installed here; ``mel_filterbank`` restates
  its published algorithm (slaney mel scale: linear below 1 kHz, logarithmic
  above; triangular filters between mel points; area normalisation);
* ``_compute_features`` (:63-88): dither, pre-emphasis ``y[0] = x[0]``,
  ``y[t] = x[t] - preemph * x[t-1]``, ``torch.stft(center=True,
  pad_mode="constant")`` (zero padding of n_fft // 2 at both ends, the window
  zero-padded to n_fft in the middle), ``|X| ** mag_power``, mel projection,
  ``log(mel + guard)``;
* ``push`` / ``_trim_samples`` (:97-151): the per-stream retained sample
  buffer, its frame bookkeeping and trimming, and the frame range a push
  emits.

The oracle keeps the reference's structure (recompute over the retained
buffer at every push) so that its frame ranges and buffer edges are the
reference's own; only the arithmetic is float64.
"""
from __future__ import annotations

import math

import numpy as np

F64 = np.float64


def hz_to_mel_slaney(f):
    """Slaney mel scale: 3 mels per 200 Hz below 1 kHz, then logarithmic with
    27 mels per factor 6.4 (librosa ``hz_to_mel(htk=False)``)."""
    f = np.asarray(f, F64)
    f_sp, min_log_hz = 200.0 / 3.0, 1000.0
    min_log_mel, logstep = min_log_hz / f_sp, math.log(6.4) / 27.0
    return np.where(f >= min_log_hz,
                    min_log_mel + np.log(np.maximum(f, 1e-300) / min_log_hz) / logstep,
                    f / f_sp)


def mel_to_hz_slaney(m):
    m = np.asarray(m, F64)
    f_sp, min_log_hz = 200.0 / 3.0, 1000.0
    min_log_mel, logstep = min_log_hz / f_sp, math.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)),
                    f_sp * m)


def mel_filterbank(sr: int, n_fft: int, n_mels: int, fmin: float, fmax: float,
                   norm: str | None = "slaney") -> np.ndarray:
    """[n_mels, 1 + n_fft // 2] float32 triangular mel filters (the published
    ``librosa.filters.mel`` algorithm, htk=False): n_mels + 2 points evenly
    spaced in slaney mels between fmin and fmax; filter i rises linearly from
    point i to point i+1 and falls to point i+2 over the FFT bin frequencies;
    ``norm="slaney"`` scales filter i by 2 / (hz[i+2] - hz[i]).  The weights
    are rounded to float32 before the normalisation, as librosa stores them."""
    fftfreqs = np.arange(1 + n_fft // 2, dtype=F64) * (1.0 / (n_fft * (1.0 / sr)))  # rfftfreq
    mel_f = mel_to_hz_slaney(np.linspace(hz_to_mel_slaney(fmin), hz_to_mel_slaney(fmax),
                                         n_mels + 2))
    fdiff = np.diff(mel_f)
    ramps = mel_f[:, None] - fftfreqs[None, :]
    w = np.empty((n_mels, fftfreqs.size), np.float32)
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        w[i] = np.maximum(0.0, np.minimum(lower, upper))
    if norm == "slaney":
        enorm = 2.0 / (mel_f[2:n_mels + 2] - mel_f[:n_mels])
        w = (w.astype(F64) * enorm[:, None]).astype(np.float32)
    elif norm is not None:
        raise ValueError(f"mel norm {norm!r} not restated")
    return w


def hann_symmetric(n: int) -> np.ndarray:
    """``torch.hann_window(n, periodic=False)``: 0.5 - 0.5 cos(2 pi i / (n - 1))."""
    if n == 1:
        return np.ones(1)
    return 0.5 - 0.5 * np.cos(2.0 * np.pi * np.arange(n, dtype=F64) / (n - 1))


class LogMel:
    """The extractor's constants and ``_compute_features`` (feature_extractor.py:
    11-88) in float64; ``dither`` is 0 unless a generator is supplied."""

    def __init__(self, sampling_rate=16000, n_mels=128, n_fft=512, window_size=0.025,
                 window_stride=0.01, preemph=0.97, log_zero_guard_value=2 ** -24,
                 lowfreq=0, highfreq=None, mag_power=2.0, mel_norm="slaney"):
        self.sr, self.n_mels, self.n_fft = sampling_rate, n_mels, n_fft
        self.win_length = int(window_size * sampling_rate)
        self.hop = int(window_stride * sampling_rate)
        self.preemph, self.guard, self.mag_power = preemph, float(log_zero_guard_value), mag_power
        w = hann_symmetric(self.win_length)
        lp = (n_fft - self.win_length) // 2                     # torch.stft centres the window
        self.window = np.zeros(n_fft)
        self.window[lp:lp + self.win_length] = w
        self.fb = mel_filterbank(sampling_rate, n_fft, n_mels, lowfreq,
                                 highfreq or sampling_rate / 2, mel_norm).astype(F64)

    def compute(self, x: np.ndarray, dither: float = 0.0, rng=None) -> np.ndarray:
        """Log-mel frames [n_mels, 1 + len(x) // hop] of one buffer."""
        x = np.asarray(x, F64)
        if dither and rng is not None:
            x = x + rng.standard_normal(x.shape) * dither
        y = np.concatenate([x[:1], x[1:] - self.preemph * x[:-1]])
        pad = self.n_fft // 2
        yp = np.concatenate([np.zeros(pad), y, np.zeros(pad)])
        nfr = 1 + (yp.size - self.n_fft) // self.hop
        idx = np.arange(nfr)[:, None] * self.hop + np.arange(self.n_fft)[None, :]
        spec = np.abs(np.fft.rfft(yp[idx] * self.window[None, :], axis=1)) ** self.mag_power
        return np.log(self.fb @ spec.T + self.guard)


class FeatureStream:
    """One stream's ``push`` state (``_fe_samples``, ``_fe_emitted_frames``,
    ``_fe_sample_offset``; parakeet/engine/sequence.py:55-57) and the
    reference's push/trim rules (feature_extractor.py:97-151)."""

    def __init__(self, mel: LogMel):
        self.mel = mel
        self.samples = np.empty((0,), np.float32)
        self.emitted = 0
        self.offset = 0

    def push(self, samples: np.ndarray, final: bool = False):
        """New frames [n_mels, F] or None, like ``FeatureExtractor.push``."""
        if not samples.size:
            return None
        self.samples = np.concatenate([self.samples, samples.astype(np.float32)])
        total = self.offset + self.samples.size
        hop, pad = self.mel.hop, self.mel.n_fft // 2
        offset_frames = self.offset // hop
        if final:
            max_frame = total // hop
        else:
            if total <= pad:
                return None
            max_frame = (total - pad) // hop
        min_frame = 0 if self.offset == 0 else (self.offset + pad + hop - 1) // hop
        start = max(self.emitted, min_frame)
        if start > max_frame:
            return None
        feats = self.mel.compute(self.samples)
        new = feats[:, start - offset_frames:max_frame - offset_frames + 1]
        self.emitted = max_frame + 1
        self._trim()
        return new

    def _trim(self):
        if self.samples.size == 0:
            return
        hop, pad = self.mel.hop, self.mel.n_fft // 2
        min_keep = max(0, self.emitted * hop - pad)
        if min_keep <= self.offset:
            return
        aligned = (min_keep // hop) * hop
        if aligned <= self.offset:
            return
        drop = aligned - self.offset
        self.samples = self.samples[drop:] if drop < self.samples.size else np.empty((0,), np.float32)
        self.offset = aligned


def frames_emitted(total_before: int, emitted_before: int, n: int, final: bool,
                   hop: int = 160, n_fft: int = 512) -> int:
    """Number of frames a push of ``n`` samples emits (feature_extractor.py:
    97-125): a non-final push emits every frame whose window ends inside the
    samples seen so far, a final push every frame up to ``total // hop``; an
    empty push emits nothing."""
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


def synth_audio(seed: int, n: int, sr: int = 16000) -> np.ndarray:
    """Seeded test audio in [-1, 1): three tones between 100 Hz and 4 kHz with
    random phases plus white noise at 20 dB SNR, quantised to pcm16 / 32768."""
    rng = np.random.default_rng(seed)
    t = np.arange(n, dtype=F64) / sr
    freqs = rng.uniform(100.0, 4000.0, 3)
    phases = rng.uniform(0.0, 2 * np.pi, 3)
    tone = sum(np.sin(2 * np.pi * f * t + p) for f, p in zip(freqs, phases)) / 3.0
    noise = rng.standard_normal(n) * (np.sqrt(np.mean(tone ** 2)) / 10.0)
    x = 0.5 * (tone + noise)
    return (np.clip(np.round(x * 32767.0), -32768, 32767) / 32768.0).astype(np.float32)


__all__ = ["LogMel", "FeatureStream", "mel_filterbank", "hann_symmetric", "frames_emitted",
           "synth_audio"]
