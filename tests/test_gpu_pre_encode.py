"""Batched streaming pre-encode on the GPU (parakeet_b200.engine.pre_encode:
the pk_pre_encode_window cache kernel through the C ABI + the ConvSubsampling
drop-in) against the reference's own outputs (tests/golden/
make_golden_pre_encode.py): rel-L2 <= 1e-5 in fp32 (TF32 off), including
first chunks shorter than the cache (the 8-frame first windows of the small
model's engine), whose streams' second windows take an 8-frame prefix."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden_pre_encode import (PRE_LARGE, PRE_SMALL, PRE_SMALL_AUDIO,  # noqa: E402
                                    chunk_frames, feature_chunk)
from parakeet_b200.engine.pre_encode import BatchedPreEncoder  # noqa: E402
from parakeet_b200.modules import ConvSubsampling  # noqa: E402
from parakeet_b200.weights import random_pre_encode_state_dict  # noqa: E402

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("cfg,name", [(PRE_SMALL, "pre_encode_small.npz"),
                                      (PRE_LARGE, "pre_encode_large.npz"),
                                      (PRE_SMALL_AUDIO, "pre_encode_small_audio.npz")])
def test_batched_pre_encode_matches_reference(cfg, name):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    g = np.load(os.path.join(HERE, "golden", name))
    m = ConvSubsampling(cfg["hidden"], cfg["channels"], cfg["feat_in"], 8)
    sd = random_pre_encode_state_dict(cfg["seed"], cfg["feat_in"], cfg["channels"], cfg["hidden"])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, strict=True)
    pe = BatchedPreEncoder(m.to("cuda").eval(), num_slots=len(cfg["streams"]),
                           cache_size=cfg["cache"], drop_extra=cfg["drop"])
    index = g["index"]
    held = {}                    # frames each stream's cache holds
    with torch.inference_mode():
        for step in sorted(set(int(s) for s in index[:, 0])):
            rows = [(int(i), bool(f)) for s, i, f in index if s == step]
            groups = {}          # rows batch together when their windows have one length
            for i, f in rows:
                groups.setdefault((f, 0 if f else held[i]), []).append(i)
            for (first, pre), group in sorted(groups.items()):
                F = chunk_frames(cfg, first)
                feats = torch.from_numpy(np.concatenate(
                    [feature_chunk(cfg, step, i, F) for i in group]))
                y = pe.pre_encode(feats, torch.tensor(group), first,
                                  prefix=None if first else pre).float().cpu().numpy()
                for r, i in enumerate(group):
                    assert rel_l2(y[r], g[f"y_{step}_{i}"]) <= 1e-5, (step, i, first)
                    held[i] = min(cfg["cache"], pre + F)
    assert int(pe.error.item()) == 0


@pytest.mark.parametrize("frames", [8, 9, 24, 25, 104, 121])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_stream_path_equals_full_path(frames, dtype):
    """forward_stream (conv1 + depthwise conv2 in one launch, conv3 depthwise,
    pointwise convs and out as GEMMs over channels-last rows, dropped rows
    skipped) against forward_full (cuDNN convs) on the same windows."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = PRE_SMALL if frames < 100 else PRE_LARGE
    m = ConvSubsampling(cfg["hidden"], cfg["channels"], cfg["feat_in"], 8)
    sd = random_pre_encode_state_dict(cfg["seed"], cfg["feat_in"], cfg["channels"], cfg["hidden"])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, strict=True)
    m = m.to("cuda", dtype).eval()
    g = torch.Generator(device="cuda").manual_seed(frames)
    xw = torch.randn(5, cfg["feat_in"], frames, generator=g, device="cuda").to(dtype)
    with torch.inference_mode():
        full = m.forward_full(xw.transpose(1, 2)).float()
        for drop in (0, 2):
            if drop >= full.shape[1]:
                continue
            got = m.forward_stream(xw, drop).float()
            ref = full[:, drop:]
            assert got.shape == ref.shape
            err = float((got - ref).norm() / ref.norm())
            assert err <= (1e-5 if dtype == torch.float32 else 2e-2), (drop, err)
