"""Golden outputs of the reference's streaming log-mel feature extractor.

Runs odunola499/parakeet-streaming's own ``FeatureExtractor``
(parakeet/modules/feature_extractor.py), imported from a source checkout
given by ``--reference``, with ``dither=0`` (the reference's dither draws
fresh ``torch.randn`` noise at every push, so only dither-free outputs are
reproducible), over seeded audio (``oracle.features.synth_audio``) pushed in
the engine's chunk sizes: a first chunk of (1 + 8 * lookahead) * hop samples,
then (8 + 8 * lookahead) * hop (parakeet/engine/model_runner.py:53-56,94-95),
plus ragged and final pushes.  ``librosa`` is stubbed with torchaudio's
slaney mel bank (``make_golden.install_librosa_stub``); that bank is saved
too, as ``fb``.  Saves ``features.npz``.

Usage:  python tests/golden/make_golden_features.py --reference <path to reference>
"""
from __future__ import annotations

import argparse
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
from make_golden import install_librosa_stub  # noqa: E402
from oracle.features import synth_audio  # noqa: E402

HOP = 160
SMALL_FIRST, SMALL_NEXT = (1 + 8 * 1) * HOP, (8 + 8 * 1) * HOP        # lookahead 1
LARGE_FIRST, LARGE_NEXT = (1 + 8 * 13) * HOP, (8 + 8 * 13) * HOP      # lookahead 13

# name -> (audio seed, [(samples, final), ...])
STREAMS = {
    "small_a": (101, [(SMALL_FIRST, False)] + [(SMALL_NEXT, False)] * 5 + [(1000, True)]),
    "small_b": (102, [(SMALL_FIRST, False)] + [(SMALL_NEXT, False)] * 3),
    "ragged": (103, [(37, False), (100, False), (300, False), (2048, False), (5, False),
                     (4000, False), (160, False), (0, False), (911, True)]),
    "tiny_final": (104, [(200, True)]),
    "large_a": (105, [(LARGE_FIRST, False), (LARGE_NEXT, False), (2000, True)]),
    "large_b": (106, [(LARGE_FIRST, False), (LARGE_NEXT, False)]),
}
FULL = {"full_3000": (107, 3000)}


def new_state():
    return SimpleNamespace(_fe_samples=np.empty((0,), np.float32), _fe_emitted_frames=0,
                           _fe_sample_offset=0)


def run():
    from parakeet.modules.feature_extractor import FeatureExtractor
    fe = FeatureExtractor(dither=0.0)
    out = {"fb": fe.fb.numpy().astype(np.float32)}
    for name, (seed, pushes) in STREAMS.items():
        audio = synth_audio(seed, sum(n for n, _ in pushes))
        st, pos, frames, counts = new_state(), 0, [], []
        for n, final in pushes:
            f = fe.push(audio[pos:pos + n], st, final=final)
            pos += n
            counts.append(0 if f is None else f.shape[-1])
            if f is not None:
                frames.append(f[0].numpy())
        out[f"{name}_feats"] = (np.concatenate(frames, axis=1) if frames
                                else np.zeros((fe.n_mels, 0), np.float32))
        out[f"{name}_counts"] = np.array(counts, np.int64)
    for name, (seed, n) in FULL.items():
        out[f"{name}_feats"] = fe(synth_audio(seed, n))[0].numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    install_librosa_stub()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "features.npz"), **run())
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
