"""The paced serving loop behind the bench's streams-at-p99 line
(bench.serve_prefill / bench.serve_trial), on CPU with a fake pipeline: the
prefill steps every position through min(age, fill) chunks; in a trial every
stream's chunks are stepped in order (first, second, later push), one chunk
per position per loop iteration; a stream that reaches its last chunk is
released and a new stream starts in its slot with a first chunk; batches never
exceed the allocator's limit; a later-chunk batch of exactly the limit goes to
the captured graph and every other batch eagerly; each measured chunk gets a
latency from its completion time."""
import os
import sys
import time

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
import bench  # noqa: E402

T, S = 2, 5


class _Event:
    def record(self, *a):
        pass

    def synchronize(self):
        pass


class _Dec:
    max_symbols = S


class FakePipe:
    device = torch.device("cpu")
    dec = _Dec()

    def __init__(self):
        self.calls = []          # (push class, slots)
        self.pushes = {}         # slot -> one list of push classes per stream it held
        self.ended = []

    def start_streams(self, slots):
        for s in torch.as_tensor(slots).tolist():
            self.pushes.setdefault(int(s), []).append([])

    def end_streams(self, slots):
        self.ended += [int(s) for s in torch.as_tensor(slots).tolist()]

    def step_audio(self, x, slots, push):
        sl = slots.tolist()
        self.calls.append((push, sl))
        for s in sl:
            self.pushes[s][-1].append(push)
        B = x.shape[0]
        time.sleep(1e-3)   # slower than the arrivals at this batch limit: batches fill up
        return torch.zeros(B, T, S, dtype=torch.int32), torch.zeros(B, T, dtype=torch.int32)


class FakeGraph:
    """Replays 'step_audio' over its own input buffers, as a captured graph does."""

    def __init__(self, pipe, xs, ss):
        self.pipe, self.xs, self.ss = pipe, xs, ss
        self.replays = 0

    def replay(self):
        self.replays += 1
        self.pipe.step_audio(self.xs, self.ss, 2)


def _bufs(cap, widths):
    hb = [torch.zeros(cap, w) for w in widths]
    db = [torch.zeros(cap, w) for w in widths]
    hs = [torch.zeros(cap, dtype=torch.int32) for _ in widths]
    ds = [torch.zeros(cap, dtype=torch.int32) for _ in widths]
    ht = [torch.zeros(cap, T * S, dtype=torch.int32) for _ in widths]
    hc = [torch.zeros(cap, T, dtype=torch.int32) for _ in widths]
    return hb, db, hs, ds, ht, hc


def _stream_ok(seg):
    """Push classes of one stream: 0, 1, then 2s (a stream may start mid-life
    after the prefill, whose chunks are in the same list)."""
    return all(c == min(j, 2) for j, c in enumerate(seg))


@pytest.mark.parametrize("use_graph", [False, True])
def test_serve_trial_steps_every_chunk_in_order(monkeypatch, use_graph):
    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: None)
    N, period, warm, meas, max_batch, life, fill = 120, 0.04, 2, 5, 2, 5, 3
    widths = (9, 16, 16)
    banks = [torch.randn(8, w) for w in widths]
    hb, db, hs, ds, ht, hc = _bufs(N, widths)
    bufs = (banks, hb, db, hs, ds, ht, hc)
    pipe = FakePipe()
    graph = None
    if use_graph:
        gx = torch.zeros(max_batch, widths[2])
        gs = torch.zeros(max_batch, dtype=torch.int32)
        graph = (FakeGraph(pipe, gx, gs), gx, gs, torch.zeros(max_batch, T, S, dtype=torch.int32),
                 torch.zeros(max_batch, T, dtype=torch.int32))
    pos = bench.ServePositions(N, period, life, fill, seed=3)
    age0 = pos.age.copy()
    bench.serve_prefill(pipe, pos, bufs, graph, max_batch=max_batch)
    for s in range(N):                     # prefill: min(age, fill) chunks, in order
        assert len(pipe.pushes[s]) == 1
        assert pipe.pushes[s][0] == [min(j, 2) for j in range(min(age0[s], fill))]
    pipe.calls.clear()
    t0 = time.perf_counter()
    lat, st = bench.serve_trial(pipe, N, pos, bufs, warm, meas, max_batch=max_batch,
                                full_graph=graph)
    elapsed = time.perf_counter() - t0
    assert elapsed < (warm + meas) * period + 2.0
    stepped = 0
    for s in range(N):
        segs = pipe.pushes[s]
        # the prefilled stream continues at its age; every later stream starts fresh
        first = [min(j, 2) for j in range(min(age0[s], fill))]
        head = segs[0][len(first):]
        assert segs[0][:len(first)] == first
        assert all(c == min(j, 2) for j, c in enumerate(head, start=age0[s])), s
        for seg in segs[1:]:
            assert _stream_ok(seg), (s, seg)
        assert len(segs) - 1 == pipe.ended.count(s)      # one release per new stream
        stepped += len(head) + sum(len(g) for g in segs[1:])
        assert len(head) + sum(len(g) for g in segs[1:]) <= warm + meas + 1
    assert st["streams_joined"] == len(pipe.ended) > 0   # lifetimes of 5 chunks: churn
    assert (pos.age >= 0).all() and (pos.age < life).all()
    assert all(len(sl) <= max_batch for _, sl in pipe.calls)
    assert all(len(sl) == len(set(sl)) for _, sl in pipe.calls)
    # chunks completing in the measured periods, each with a non-negative latency
    # (how many were stepped depends on the host's speed: the loop runs in real time)
    assert 0 < lat.size <= N * (meas + 1)
    assert (lat >= 0).all()
    assert st["backlog_chunks_at_end"] >= 0
    assert st["steps"] == len(pipe.calls)
    full = [sl for c, sl in pipe.calls if c == 2 and len(sl) == max_batch]
    assert full, "the trial should have made full later-chunk batches"
    if use_graph:   # exactly those went through the graph (its input buffers)
        assert graph[0].replays >= len(full)
    else:
        assert all(c != 2 or len(sl) <= max_batch for c, sl in pipe.calls)
