"""Batched greedy RNNT decode on the GPU (parakeet_b200.engine.decoding, through
the pk_rnnt_pick / pk_lstm_cell C ABI) against the token ids the reference's
ModelRunner._decode_batch produced on the same seeded inputs
(tests/golden/make_golden_decode.py): identical in fp32."""
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden_decode import DECODE_LARGE, DECODE_SMALL, decode_chunk  # noqa: E402
from parakeet_b200.engine.decoding import BatchedGreedyDecoder  # noqa: E402
from parakeet_b200.modules import Joiner, Predictor  # noqa: E402
from parakeet_b200.weights import random_decoder_state_dict  # noqa: E402

pytestmark = pytest.mark.gpu


def build(cfg, dtype):
    pred = Predictor(cfg["pred_dim"], cfg["pred_dim"], cfg["pred_layers"], cfg["vocab"])
    join = Joiner(cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"], num_classes=cfg["vocab"])
    sd = random_decoder_state_dict(cfg["seed"], cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"],
                                   cfg["vocab"], cfg["pred_layers"], cfg["blank_bias"])
    pred.load_state_dict({k[10:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("predictor.")}, strict=True)
    join.load_state_dict({k[7:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("joiner.")}, strict=True)
    return pred.to("cuda", dtype).eval(), join.to("cuda", dtype).eval()


def replay(cfg, dtype):
    torch.backends.cuda.matmul.allow_tf32 = False
    pred, join = build(cfg, dtype)
    dec = BatchedGreedyDecoder(pred, join, cfg["vocab"], num_slots=len(cfg["streams"]),
                               max_symbols=cfg["max_symbols"])
    seen, out = set(), []
    with torch.inference_mode():
        for step in range(cfg["steps"]):
            seqs, chunks, keys = [], [], []
            for i, (name, first, lens) in enumerate(cfg["streams"]):
                if step < first:
                    continue
                if i not in seen:
                    dec.reset_slots([i])
                    seen.add(i)
                length = (lens or {}).get(step, cfg["chunk"])
                seqs.append(SimpleNamespace(encoder_state=i))
                chunks.append(torch.from_numpy(decode_chunk(cfg, step, i, length)))
                keys.append((step, i, length))
            out += list(zip(keys, dec.decode_batch(seqs, chunks)))
    return out


def golden(name):
    g = np.load(os.path.join(HERE, "golden", name))
    t, off, index = g["tokens"], g["offsets"], g["index"]
    return [(tuple(index[i]), list(t[off[i]:off[i + 1]])) for i in range(len(index))]


@pytest.mark.parametrize("cfg,name", [(DECODE_SMALL, "decode_small.npz"),
                                      (DECODE_LARGE, "decode_large.npz")])
def test_batched_greedy_decode_matches_reference_fp32(cfg, name):
    got, want = replay(cfg, torch.float32), golden(name)
    assert [k for k, _ in got] == [k for k, _ in want]
    for (k, a), (_, b) in zip(got, want):
        assert a == b, (k, a, b)


def test_batched_greedy_decode_bf16_runs():
    got = replay(DECODE_SMALL, torch.bfloat16)
    n = sum(len(t) for _, t in got)
    assert 0 < n <= sum(k[2] for k, _ in got) * DECODE_SMALL["max_symbols"]
    assert all(0 <= x < DECODE_SMALL["vocab"] for _, t in got for x in t)
