"""Golden token ids of the reference engine end to end.

Runs odunola499/parakeet-streaming's own ``ModelRunner.step()``
(parakeet/engine/model_runner.py:103-107: pre-encode with the reference's
``FeatureExtractor.push`` and ``ConvSubsampling``, the batched encode step over
its ``Scheduler`` pool, the greedy RNNT decode), imported from a source checkout
given by ``--reference``, synchronously on the CPU in fp32, one stream: 10 s of
pcm16 white noise (seed 0, amplitude uniform in +-8000) pushed in 160 ms pieces
(``tests/engine_drive.py``).  Saved per model size as ``e2e_<size>.npz``: the
token ids of every encoder chunk, the chunk's frame count and the encoder
output (full depth: 17 layers small, 24 large), plus the smallest gap between
the two largest joint logits over every greedy decision (how far the argmax
is from a tie, for reading a failure).

Shims (the reference cannot download weights or import librosa offline):
``baseline/harness.py``: ``librosa.filters.mel`` is torchaudio's slaney bank;
``Parakeet.from_pretrained`` returns a ``Parakeet`` built from the config and
loaded with ``parakeet_b200.weights.random_model_state_dict`` (seed 0), whose
``_feature_extractor`` is ``FeatureExtractor(dither=0.0)`` (dither draws from
the global RNG, feature_extractor.py:66) and ``_tokenizer`` a stub.

Usage:  python tests/golden/make_golden_e2e.py --reference <path to reference>
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "parakeet-streaming_b200"))
sys.path.insert(0, os.path.join(REPO, "tests"))
sys.path.insert(0, os.path.join(REPO, "baseline"))
import harness  # noqa: E402
from engine_drive import drive, pack, pcm16_noise  # noqa: E402

# Weights: harness.MODEL_WEIGHTS (seed 0; blank_bias 2.3 small, 1.0 large, so
# that the random joint emits 0-5 symbols per frame instead of always 5 or
# never: small 286 tokens over 128 frames, large 100 over 140).  Audio:
# configs[0], pushed in 160 ms pieces.
AUDIO = dict(audio_seed=0, seconds=10.0, push=2560)


def reference_runner(size, device="cpu", dtype=torch.float32, max_streams=2):
    """The reference's ModelRunner over its own modules and seeded weights."""
    from parakeet.config import Config
    from parakeet.engine.model_runner import ModelRunner
    from parakeet.engine.scheduler import Scheduler

    harness.patch_from_pretrained(harness.seeded_parakeet(size, dtype))
    conf = Config(size=size, max_num_streams=max_streams)
    return ModelRunner(conf, torch.device(device), Scheduler(max_active=max_streams))


def run(size):
    cfg = AUDIO
    runner = reference_runner(size)
    gaps = []

    def margin(_m, _inp, out):
        top = out.float().topk(2, dim=-1).values
        gaps.append(float((top[..., 0] - top[..., 1]).min()))

    runner.joiner.register_forward_hook(margin)
    audio = pcm16_noise(cfg["audio_seed"], cfg["seconds"])
    t0 = time.perf_counter()
    rec = drive(runner, audio, cfg["push"])
    dt = time.perf_counter() - t0
    out = pack(rec)
    out["min_margin"] = np.array(min(gaps))
    out["blank"] = np.array(harness.MODEL_WEIGHTS[size]["vocab"])
    nb = len(out["tokens"])
    print(f"{size}: {len(rec)} chunks, {int(out['frames'].sum())} frames, {nb} tokens, "
          f"{len(gaps)} joint calls, min top-2 gap {min(gaps):.3e}, {dt:.1f} s")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--sizes", default="small,large")
    args = ap.parse_args()
    harness.import_reference(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for size in args.sizes.split(","):
        np.savez_compressed(os.path.join(HERE, f"e2e_{size}.npz"), **run(size))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
