"""Loads the reference (odunola499/parakeet-streaming) for the reference arm
of ``bench.py`` and the engine-level drop-in tests.

The reference is pure Python; ``bench.py --install-reference <checkout>``
places it under ``baseline/_ref`` (git-ignored, travels with the working tree).
Nothing here is part of the product: the package never imports it.

Two shims make the reference run offline, without changing its code:
* ``librosa`` (imported at the top of parakeet/modules/feature_extractor.py:3)
  is absent: a stub ``librosa.filters.mel`` returns torchaudio's slaney mel
  bank (the same bank, torchaudio implements librosa's slaney formula);
* HF weights cannot be downloaded: ``Parakeet.from_pretrained``
  (parakeet/model.py:107-130) is replaced by a function that returns a
  ``Parakeet`` built from the config and loaded with seeded weights
  (``parakeet_b200.weights.random_model_state_dict``), with the reference's
  ``FeatureExtractor`` and a stub tokenizer.
"""
from __future__ import annotations

import os
import sys
import types
from types import SimpleNamespace

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")


def install_librosa_stub() -> None:
    try:
        import librosa  # noqa: F401
        return
    except ImportError:
        pass
    import torchaudio

    lib = types.ModuleType("librosa")
    filters = types.ModuleType("librosa.filters")

    def mel(sr, n_fft, n_mels, fmin, fmax, norm):
        fb = torchaudio.functional.melscale_fbanks(
            n_fft // 2 + 1, float(fmin), float(fmax), n_mels, sr,
            norm=norm, mel_scale="slaney")
        return fb.T.numpy()

    filters.mel = mel
    lib.filters = filters
    sys.modules["librosa"] = lib
    sys.modules["librosa.filters"] = filters


def available(path: str | None = None) -> bool:
    return os.path.isfile(os.path.join(path or REF_DIR, "parakeet", "engine", "model_runner.py"))


def import_reference(path: str | None = None):
    """Makes ``import parakeet`` resolve to the reference at ``path``
    (default ``baseline/_ref``) and returns the package."""
    path = os.path.abspath(path or REF_DIR)
    if not available(path):
        raise FileNotFoundError(f"no reference install at {path}")
    install_librosa_stub()
    if path not in sys.path:
        sys.path.insert(0, path)
    import parakeet
    return parakeet


# Seeded weights of the end-to-end runs: the reference's ModelConfig /
# LargeModelConfig shapes (parakeet/config.py:5-31); blank_bias shifts the
# blank logit so that the random joint emits 0-5 symbols per frame.
MODEL_WEIGHTS = {
    "small": dict(layers=17, dim=512, heads=8, vocab=1026, pred_layers=1, seed=0, blank_bias=2.3),
    "large": dict(layers=24, dim=1024, heads=8, vocab=1024, pred_layers=2, seed=0, blank_bias=1.0),
}


def model_state_dict(size: str):
    from parakeet_b200.weights import random_model_state_dict
    c = MODEL_WEIGHTS[size]
    return random_model_state_dict(c["seed"], c["layers"], c["dim"], c["heads"], c["vocab"],
                                   c["pred_layers"], blank_bias=c["blank_bias"])


def seeded_parakeet(size: str, dtype=None):
    """The reference's ``Parakeet`` for ``size`` with the seeded weights, its
    own ``FeatureExtractor(dither=0.0)`` and a stub tokenizer."""
    import torch
    from parakeet.config import Config
    from parakeet.model import Parakeet
    from parakeet.modules import FeatureExtractor

    torch.manual_seed(0)
    model = Parakeet(Config(size=size).model_config)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in model_state_dict(size).items()},
                          strict=True)
    model._feature_extractor = FeatureExtractor(dither=0.0)
    model._tokenizer = SimpleNamespace(decode=lambda ids: "")
    return model.to(dtype) if dtype is not None else model


def patch_from_pretrained(model) -> None:
    """``Parakeet.from_pretrained`` returns ``model`` (no download)."""
    from parakeet.model import Parakeet
    Parakeet.from_pretrained = classmethod(lambda cls, size="small": model)
