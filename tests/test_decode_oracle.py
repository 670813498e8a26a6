"""The greedy RNNT decode restatement (oracle/decode.py) against the token ids
the reference's own ModelRunner._decode_batch produced on the same seeded
inputs (tests/golden/make_golden_decode.py)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "parakeet-streaming_b200"))
from make_golden_decode import DECODE_LARGE, DECODE_SMALL, decode_chunk  # noqa: E402
from oracle.decode import GreedyDecoderModel  # noqa: E402
from parakeet_b200.weights import random_decoder_state_dict  # noqa: E402


def golden_lists(name):
    g = np.load(os.path.join(HERE, "golden", name))
    toks, off, index = g["tokens"], g["offsets"], g["index"]
    return [(tuple(index[i]), list(toks[off[i]:off[i + 1]])) for i in range(len(index))]


def oracle_lists(cfg):
    sd = random_decoder_state_dict(cfg["seed"], cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"],
                                   cfg["vocab"], cfg["pred_layers"], cfg["blank_bias"])
    m = GreedyDecoderModel(sd, cfg["pred_layers"], cfg["vocab"], cfg["max_symbols"])
    state, out = {}, []
    for step in range(cfg["steps"]):
        for i, (name, first, lens) in enumerate(cfg["streams"]):
            if step < first:
                continue
            if name not in state:
                state[name] = m.new_stream()
            length = (lens or {}).get(step, cfg["chunk"])
            toks, po, st = m.decode_chunk(decode_chunk(cfg, step, i, length)[0], *state[name])
            state[name] = (po, st)
            out.append(((step, i, length), toks))
    return out


@pytest.mark.parametrize("cfg,name", [(DECODE_SMALL, "decode_small.npz"),
                                      (DECODE_LARGE, "decode_large.npz")])
def test_oracle_decode_matches_reference_tokens(cfg, name):
    got, want = oracle_lists(cfg), golden_lists(name)
    assert [k for k, _ in got] == [k for k, _ in want]
    for (k, a), (_, b) in zip(got, want):
        assert a == b, (k, a, b)
    assert sum(len(t) for _, t in want) > 50   # blanks and tokens both occur


def test_drop_in_modules_load_reference_state_dict_keys():
    """The Predictor / Joiner drop-ins take the reference's parameter names."""
    import torch
    from parakeet_b200.modules import Joiner, Predictor
    cfg = DECODE_LARGE
    sd = random_decoder_state_dict(1, cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"],
                                   cfg["vocab"], cfg["pred_layers"])
    pred = Predictor(cfg["pred_dim"], cfg["pred_dim"], cfg["pred_layers"], cfg["vocab"])
    join = Joiner(cfg["enc_dim"], cfg["pred_dim"], cfg["joint_dim"], num_classes=cfg["vocab"])
    pred.load_state_dict({k[10:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("predictor.")}, strict=True)
    join.load_state_dict({k[7:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("joiner.")}, strict=True)
