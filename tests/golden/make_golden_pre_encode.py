"""Golden outputs of the reference's streaming pre-encoder.

Runs odunola499/parakeet-streaming's own ``ConvSubsampling``
(parakeet/modules/subsample.py), imported from a source checkout given by
``--reference``, with ``parakeet_b200.weights.random_pre_encode_state_dict``,
on seeded feature chunks of several streams, with the per-stream cache
handling of ``ModelRunner._run_pre_encode`` (parakeet/engine/model_runner.py:
197-233, restated here because the runner method also drives the feature
extractor): feats_in = cat(cache, feats) when a cache exists, subsample, drop
the first ``drop_extra_pre_encoded`` output frames when a cache was used,
cache = last ``pre_encode_cache_size`` frames of feats_in.  First chunks have
1 + 8 * lookahead feature frames, later ones 8 + 8 * lookahead
(model_runner.py:53-56); ``PRE_SMALL_AUDIO`` has the 8-frame first chunks that
the feature extractor emits from a first chunk of samples, shorter than the
cache, which then holds the whole first window.  Saves
``pre_encode_small.npz`` / ``_large.npz`` / ``_small_audio.npz``.

Usage:  python tests/golden/make_golden_pre_encode.py --reference <path to reference>
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "parakeet-streaming_b200"))
sys.path.insert(0, HERE)
from make_golden import install_librosa_stub  # noqa: E402
from parakeet_b200.weights import random_pre_encode_state_dict, seeded_normal  # noqa: E402

PRE_SMALL = dict(feat_in=128, channels=256, hidden=512, lookahead=1, cache=9, drop=2, seed=41,
                 steps=4, streams=[("a", 0), ("b", 0), ("c", 2)])
PRE_LARGE = dict(feat_in=128, channels=256, hidden=1024, lookahead=13, cache=9, drop=2, seed=42,
                 steps=3, streams=[("a", 0), ("b", 1)])
# first chunks as the feature extractor emits them from 1 + 8 * lookahead hops of
# samples: 8 * lookahead frames, fewer than the cache for lookahead 1
PRE_SMALL_AUDIO = dict(PRE_SMALL, seed=43, first_frames=8)


def chunk_frames(cfg, first):
    if first:
        return cfg.get("first_frames", 1 + 8 * cfg["lookahead"])
    return 8 + 8 * cfg["lookahead"]


def feature_chunk(cfg, step, i, frames):
    """Feature chunk [1, feat_in, frames] of one stream and step."""
    return seeded_normal(cfg["seed"] * 100000 + step * 100 + i, (1, cfg["feat_in"], frames))


def run(cfg):
    from parakeet.modules.subsample import ConvSubsampling
    m = ConvSubsampling(cfg["hidden"], cfg["channels"], cfg["feat_in"], 8)
    sd = random_pre_encode_state_dict(cfg["seed"], cfg["feat_in"], cfg["channels"], cfg["hidden"])
    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()}, strict=True)
    m.eval()
    caches, out, index = {}, {}, []
    with torch.inference_mode():
        for step in range(cfg["steps"]):
            for i, (name, first_step) in enumerate(cfg["streams"]):
                if step < first_step:
                    continue
                first = name not in caches
                feats = torch.from_numpy(feature_chunk(cfg, step, i, chunk_frames(cfg, first)))
                cache = caches.get(name)
                x = feats if cache is None else torch.cat([cache, feats], dim=-1)
                lengths = torch.full((1,), x.size(-1), dtype=torch.int64)
                y, _ = m(x.transpose(1, 2), lengths)
                if cache is not None and cfg["drop"] > 0:
                    y = y[:, cfg["drop"]:, :]
                caches[name] = x[:, :, -cfg["cache"]:] if x.size(-1) >= cfg["cache"] else x
                out[f"y_{step}_{i}"] = y[0].numpy()
                index.append((step, i, int(first)))
    out["index"] = np.array(index, np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    install_librosa_stub()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "pre_encode_small.npz"), **run(PRE_SMALL))
    np.savez_compressed(os.path.join(HERE, "pre_encode_large.npz"), **run(PRE_LARGE))
    np.savez_compressed(os.path.join(HERE, "pre_encode_small_audio.npz"), **run(PRE_SMALL_AUDIO))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
