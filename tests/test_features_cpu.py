"""Streaming log-mel features on the CPU: the float64 oracle (oracle/features.py)
against the reference extractor's own outputs (tests/golden/
make_golden_features.py), and the host side of the GPU extractor (the
C-ABI's constant tables and the frame-count rule) against the oracle."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden_features import FULL, STREAMS  # noqa: E402
from oracle.features import (FeatureStream, LogMel, frames_emitted as oracle_frames,  # noqa: E402
                             hann_symmetric, mel_filterbank, synth_audio)

GOLD = np.load(os.path.join(HERE, "golden", "features.npz"))
# log-mel, absolute: float64 oracle vs the reference's float32 torch.stft path
LOGMEL_TOL = 2e-3


def run_oracle(pushes, seed):
    audio = synth_audio(seed, sum(n for n, _ in pushes))
    st, pos, frames, counts = FeatureStream(LogMel()), 0, [], []
    for n, final in pushes:
        f = st.push(audio[pos:pos + n], final)
        pos += n
        counts.append(0 if f is None else f.shape[1])
        if f is not None:
            frames.append(f)
    return (np.concatenate(frames, 1) if frames else np.zeros((128, 0))), counts


@pytest.mark.parametrize("name", sorted(STREAMS))
def test_oracle_push_matches_reference(name):
    seed, pushes = STREAMS[name]
    got, counts = run_oracle(pushes, seed)
    assert counts == list(GOLD[f"{name}_counts"])
    ref = GOLD[f"{name}_feats"]
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= LOGMEL_TOL


def test_oracle_whole_utterance_matches_reference():
    for name, (seed, n) in FULL.items():
        got = LogMel().compute(synth_audio(seed, n))
        ref = GOLD[f"{name}_feats"]
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= LOGMEL_TOL


def test_oracle_filterbank_matches_reference_bank():
    """The restated librosa slaney bank against the bank the golden run used
    (torchaudio's slaney implementation, float32)."""
    fb = mel_filterbank(16000, 512, 128, 0.0, 8000.0)
    ref = GOLD["fb"]
    assert fb.shape == ref.shape == (128, 257)
    assert np.abs(fb - ref).max() <= 1e-6
    assert ((fb > 0) == (ref > 0)).mean() > 0.995


def test_frame_count_rule_matches_reference():
    from parakeet_b200.modules.features import frames_emitted
    for name, (seed, pushes) in STREAMS.items():
        seen = emitted = 0
        got = []
        for n, final in pushes:
            c = frames_emitted(seen, emitted, n, final, 160, 512)
            assert c == oracle_frames(seen, emitted, n, final)
            got.append(c)
            seen += n
            emitted += c
        assert got == list(GOLD[f"{name}_counts"]), name


def _tables_extractor(**kw):
    from parakeet_b200.modules.features import FeatureExtractor
    return FeatureExtractor(device="cpu", **kw)


def test_c_abi_tables_match_oracle():
    """pk_features_tables (host code of libpk.so) builds the same filter bank
    and window as the oracle's restatement."""
    fe = _tables_extractor()
    fb = fe.fb.numpy()
    ref = mel_filterbank(16000, 512, 128, 0.0, 8000.0)
    assert fb.shape == ref.shape
    assert np.abs(fb - ref).max() <= 1e-7 * max(1.0, np.abs(ref).max())
    assert fe.mel_nnz == int((ref != 0).sum())
    words = fe.tables.numpy()
    assert words[0] == 0x45464b50 and words[1] == 512 and words[2] == 128
    tw = words[16:16 + 1024].view(np.float32).reshape(512, 2)
    u = np.arange(512)
    assert np.abs(tw[:, 0] - np.cos(2 * np.pi * u / 512)).max() < 1e-7
    assert np.abs(tw[:, 1] + np.sin(2 * np.pi * u / 512)).max() < 1e-7
    win = words[16 + 1024:16 + 1536].view(np.float32)
    ref_win = np.zeros(512)
    ref_win[56:456] = hann_symmetric(400)
    assert np.abs(win - ref_win).max() < 1e-7


def test_c_abi_tables_other_configs():
    fe = _tables_extractor(n_mels=80, mel_norm=None, lowfreq=20, highfreq=7600)
    ref = mel_filterbank(16000, 512, 80, 20.0, 7600.0, norm=None)
    assert np.abs(fe.fb.numpy() - ref).max() <= 1e-7


def test_c_abi_tables_reject_bad_arguments():
    from parakeet_b200._lib import PKError
    with pytest.raises(PKError):
        _tables_extractor(n_mels=300)
    with pytest.raises(PKError):
        _tables_extractor(highfreq=9000)
    with pytest.raises(ValueError):
        _tables_extractor(mel_norm="htk")


def test_push_needs_a_cuda_device():
    fe = _tables_extractor(num_slots=2)
    with pytest.raises(RuntimeError, match="CUDA"):
        fe.push_batch(np.zeros((1, 1600), np.float32), [0], first=True)
