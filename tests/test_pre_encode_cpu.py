"""The ConvSubsampling drop-in (parakeet_b200.modules.subsample) against the
reference's own pre-encoder outputs (tests/golden/make_golden_pre_encode.py),
on the CPU with the per-stream cache handling of _run_pre_encode."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden_pre_encode import (PRE_LARGE, PRE_SMALL, PRE_SMALL_AUDIO,  # noqa: E402
                                    chunk_frames, feature_chunk)
from parakeet_b200.modules import ConvSubsampling  # noqa: E402
from parakeet_b200.weights import random_pre_encode_state_dict  # noqa: E402


def build(cfg):
    m = ConvSubsampling(cfg["hidden"], cfg["channels"], cfg["feat_in"], 8)
    sd = random_pre_encode_state_dict(cfg["seed"], cfg["feat_in"], cfg["channels"], cfg["hidden"])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, strict=True)
    return m.eval()


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("cfg,name", [(PRE_SMALL, "pre_encode_small.npz"),
                                      (PRE_LARGE, "pre_encode_large.npz"),
                                      (PRE_SMALL_AUDIO, "pre_encode_small_audio.npz")])
def test_subsampling_drop_in_matches_reference(cfg, name):
    g = np.load(os.path.join(HERE, "golden", name))
    m = build(cfg)
    caches = {}
    with torch.inference_mode():
        for step, i, first in g["index"]:
            feats = torch.from_numpy(feature_chunk(cfg, step, i, chunk_frames(cfg, bool(first))))
            c = caches.get(i)
            x = feats if c is None else torch.cat([c, feats], -1)
            y, _ = m(x.transpose(1, 2), torch.full((1,), x.size(-1), dtype=torch.int64))
            if c is not None:
                y = y[:, cfg["drop"]:]
            caches[i] = x[:, :, -cfg["cache"]:]
            assert rel_l2(y[0].numpy(), g[f"y_{step}_{i}"]) <= 1e-5, (step, i)


def test_subsampling_masks_frames_beyond_length():
    """Rows shorter than the batch: frames at or beyond a row's length do not
    change its output (MaskedConvSequential semantics)."""
    m = build(PRE_SMALL)
    x = torch.randn(2, 25, 128)
    y_full, l_full = m(x[1:2, :17], torch.tensor([17]))
    x2 = x.clone()
    x2[1, 17:] = 1e3
    y, lens = m(torch.stack([x[0], x2[1]])[:, :25], torch.tensor([25, 17]))
    assert lens.tolist() == [4, l_full.item()]
    assert torch.allclose(y[1, : l_full.item()], y_full[0], rtol=1e-4, atol=1e-5)


def test_full_length_path_equals_masked_forward():
    m = build(PRE_SMALL)
    x = torch.randn(3, 25, 128)
    with torch.inference_mode():
        y, _ = m(x, torch.full((3,), 25))
        y2 = m.forward_full(x)
    assert torch.allclose(y, y2, rtol=1e-5, atol=1e-5)
