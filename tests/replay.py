"""Replays the golden stream schedules (tests/golden/make_golden.py) against
any implementation: the oracle here, the CUDA path in the GPU tests."""
from __future__ import annotations

import importlib.util
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_spec = importlib.util.spec_from_file_location(
    "make_golden", os.path.join(HERE, "golden", "make_golden.py"))
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)

SMALL = make_golden.SMALL_SCHEDULE
LARGE = make_golden.LARGE_SCHEDULE
SMALL_FULL = make_golden.SMALL_FULL
LARGE_FULL = make_golden.LARGE_FULL


def load(name):
    return dict(np.load(os.path.join(HERE, "golden", name)))


def schedule(cfg):
    """Yields (step, releases, acquires, batch names, x [B,T,D] f32, lengths)."""
    T = cfg["att"][1] + 1
    for s, batch in enumerate(make_golden.schedule_batches(cfg)):
        rel = [e[0] for e in cfg["events"] if e[2] == s]
        acq = [e[0] for e in cfg["events"] if e[1] == s]
        x = make_golden.encoder_stream_inputs(cfg["seed"], s, len(batch), T, cfg["dim"])
        yield s, rel, acq, [n for n, _ in batch], x, np.array([n for _, n in batch])


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def valid_rows(out_bdt, lengths):
    """Concatenate the valid time columns of a [B, D, T] output."""
    return np.concatenate([out_bdt[b, :, :int(n)].ravel() for b, n in enumerate(lengths)])
