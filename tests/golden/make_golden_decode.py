"""Golden token ids of the reference's batched greedy RNNT decode.

Runs ``ModelRunner._decode_batch`` / ``_decode_frame_batch``
(parakeet/engine/model_runner.py:347-447) of odunola499/parakeet-streaming,
imported from a source checkout given by ``--reference``, on seeded encoder
outputs with ragged chunk lengths, and saves the emitted token ids per
(step, stream) as ``decode_small.npz``.  The prediction and joint networks are
the reference's own ``Predictor`` and ``Joiner`` (parakeet/modules/decoder.py)
loaded with ``parakeet_b200.weights.random_decoder_state_dict``; the runner
method is called on a plain object that carries the attributes it reads
(``joiner``, ``decoder``, ``blank_id``, ``_max_symbols_per_frame`` and its
helper methods), since a full ``ModelRunner`` needs a tokenizer and weights
from the network.  Per-stream state starts as in ``create_sequence``
(model_runner.py:66-80): zeros, then one prediction step on the blank id.

Usage:  python tests/golden/make_golden_decode.py --reference <path to reference>
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
sys.path.insert(0, os.path.join(REPO, "parakeet-streaming_b200"))
sys.path.insert(0, HERE)
from make_golden import install_librosa_stub  # noqa: E402
from parakeet_b200.weights import random_decoder_state_dict, seeded_normal  # noqa: E402

# (name, first step, chunk length per step or None for full chunks).  Streams are
# handed to the batch in this order; lengths are ragged so that _decode_batch's
# sort-by-length and shrinking active batch are exercised.
DECODE_SMALL = dict(enc_dim=512, pred_dim=640, joint_dim=640, vocab=1026, pred_layers=1,
                    chunk=2, steps=6, seed=31, blank_bias=2.3, max_symbols=5,
                    streams=[("a", 0, None), ("b", 0, {2: 1}), ("c", 1, None),
                             ("d", 2, {4: 1}), ("e", 3, None)])
DECODE_LARGE = dict(enc_dim=1024, pred_dim=640, joint_dim=640, vocab=1024, pred_layers=2,
                    chunk=14, steps=3, seed=32, blank_bias=2.3, max_symbols=5,
                    streams=[("a", 0, None), ("b", 0, {1: 9}), ("c", 1, None)])


def build(cfg):
    from parakeet.modules.decoder import Joiner, Predictor
    pred = Predictor(cfg["pred_dim"], cfg["pred_dim"], cfg["pred_layers"], cfg["vocab"])
    join = Joiner(cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"], num_classes=cfg["vocab"])
    sd = random_decoder_state_dict(cfg["seed"], cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"],
                                   cfg["vocab"], cfg["pred_layers"], cfg["blank_bias"])
    pred.load_state_dict({k[len("predictor."):]: torch.from_numpy(v)
                          for k, v in sd.items() if k.startswith("predictor.")}, strict=True)
    join.load_state_dict({k[len("joiner."):]: torch.from_numpy(v)
                          for k, v in sd.items() if k.startswith("joiner.")}, strict=True)
    return pred.eval(), join.eval()


def decode_chunk(cfg, step, name_idx, length):
    """Encoder output chunk [1, enc_dim, length] of one stream and step."""
    x = seeded_normal(cfg["seed"] * 100000 + step * 100 + name_idx, (1, cfg["enc_dim"], cfg["chunk"]))
    return x[:, :, :length]


def run(cfg):
    from parakeet.engine.model_runner import ModelRunner
    pred, join = build(cfg)
    blank = cfg["vocab"]
    runner = SimpleNamespace(joiner=join, decoder=pred, blank_id=blank,
                             _max_symbols_per_frame=cfg["max_symbols"])
    runner._stack_states = lambda states: ModelRunner._stack_states(runner, states)
    runner._unstack_states = lambda sb: ModelRunner._unstack_states(runner, sb)
    runner._decode_frame_batch = lambda f, p, s: ModelRunner._decode_frame_batch(runner, f, p, s)
    seqs = {}
    out = {"blank": np.array(blank)}
    tokens, offsets, index = [], [0], []
    with torch.inference_mode():
        for step in range(cfg["steps"]):
            batch, chunks = [], []
            for i, (name, first, lens) in enumerate(cfg["streams"]):
                if step < first:
                    continue
                if name not in seqs:   # create_sequence, model_runner.py:66-80
                    st = pred.init_state(1)
                    po, st = pred(torch.full((1,), blank, dtype=torch.long), state=st)
                    seqs[name] = SimpleNamespace(pred_out=po, pred_state=st)
                length = (lens or {}).get(step, cfg["chunk"])
                batch.append(seqs[name])
                chunks.append(torch.from_numpy(decode_chunk(cfg, step, i, length)))
                index.append((step, i, length))
            lists = ModelRunner._decode_batch(runner, batch, chunks)
            for toks in lists:
                tokens.extend(toks)
                offsets.append(len(tokens))
    out["tokens"] = np.array(tokens, np.int64)
    out["offsets"] = np.array(offsets, np.int64)
    out["index"] = np.array(index, np.int64)   # (step, stream, length) per token list
    nonblank = len(tokens)
    frames = int(sum(l for _, _, l in index))
    print(f"{len(index)} stream-chunks, {frames} frames, {nonblank} tokens "
          f"({nonblank / max(1, frames):.2f} per frame, max {cfg['max_symbols']})")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    install_librosa_stub()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    np.savez_compressed(os.path.join(HERE, "decode_small.npz"), **run(DECODE_SMALL))
    np.savez_compressed(os.path.join(HERE, "decode_large.npz"), **run(DECODE_LARGE))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
