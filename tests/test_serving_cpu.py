"""The paced serving loop behind the bench's streams-at-p99 line
(bench.serve_prefill / bench.serve_trial), on CPU with a fake pipeline: the
prefill steps every position through min(age, fill) chunks; in a trial every
stream's chunks are stepped in order (first, second, later push), one chunk
per position per loop iteration; a stream that reaches its last chunk is
released and a new stream starts in its slot with a first chunk; batches never
exceed the loop's limit; with step graphs every batch is cut into bucket-sized
replays, the last padded with spare slots, and the released streams' pages are
returned (a step start of no rows) before the next replay; each measured chunk
gets a latency from its completion time."""
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


class FakePool:
    def __init__(self):
        self.pending_release = []
        self.flushes = 0

    def begin_step(self, slots, *a, **k):
        assert slots.numel() == 0
        self.pending_release = []
        self.flushes += 1


class FakePipe:
    device = torch.device("cpu")
    dec = _Dec()

    def __init__(self, check_flushed=False):
        self.calls = []          # (push class, slots)
        self.pushes = {}         # slot -> one list of push classes per stream it held
        self.ended = []
        self.pool = FakePool()
        self.check_flushed = check_flushed

    def start_streams(self, slots):
        for s in torch.as_tensor(slots).tolist():
            self.pushes.setdefault(int(s), []).append([])

    def end_streams(self, slots):
        sl = [int(s) for s in torch.as_tensor(slots).tolist()]
        self.ended += sl
        self.pool.pending_release += sl

    def step_audio(self, x, slots, push):
        if self.check_flushed:   # a replayed step carries no releases
            assert not self.pool.pending_release
        sl = slots.tolist()
        self.calls.append((push, sl))
        for s in sl:
            self.pushes[s][-1].append(push)
        B = x.shape[0]
        time.sleep(1e-3)   # slower than the arrivals at this batch limit: batches fill up
        return torch.zeros(B, T, S, dtype=torch.int32), torch.zeros(B, T, dtype=torch.int32)


class FakeGraph:
    """Replays 'step_audio' over its own input buffers, as a captured graph does."""

    def __init__(self, pipe, xs, ss, push):
        self.pipe, self.xs, self.ss, self.push = pipe, xs, ss, push
        self.replays = 0

    def replay(self):
        self.replays += 1
        self.pipe.step_audio(self.xs, self.ss, self.push)


class FakeStepGraphs(bench.StepGraphs):
    """bench.StepGraphs' batching over fake graphs of small buckets."""

    def __init__(self, pipe, sizes, dummy, widths):
        self.dummy = torch.tensor(dummy, dtype=torch.int32)
        self.sizes = sorted(sizes, reverse=True)
        self.g = {}
        for c in range(3):
            for Bg in sizes:
                gx, gs = torch.zeros(Bg, widths[c]), torch.zeros(Bg, dtype=torch.int32)
                self.g[(c, Bg)] = (FakeGraph(pipe, gx, gs, c), gx, gs,
                                   torch.zeros(Bg, T, S, dtype=torch.int32),
                                   torch.zeros(Bg, T, dtype=torch.int32))
        pipe.start_streams(self.dummy)


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
    N, period, warm, meas, max_batch, life, fill = 120, 0.04, 2, 5, 5, 5, 3
    widths = (9, 16, 16)
    banks = [torch.randn(8, w) for w in widths]
    hb, db, hs, ds, ht, hc = _bufs(N, widths)
    bufs = (banks, hb, db, hs, ds, ht, hc)
    pipe = FakePipe(check_flushed=use_graph)
    graph = FakeStepGraphs(pipe, (4, 2), [N, N + 1], widths) if use_graph else None
    pos = bench.ServePositions(N, period, life, fill, seed=3)
    age0 = pos.age.copy()
    bench.serve_prefill(pipe, pos, bufs, graph, max_batch=max_batch)
    for s in range(N):                     # prefill: min(age, fill) chunks, in order
        assert len(pipe.pushes[s]) == 1
        assert pipe.pushes[s][0] == [min(j, 2) for j in range(min(age0[s], fill))]
    pipe.calls.clear()
    replays0 = sum(g[0].replays for g in graph.g.values()) if use_graph else 0
    t0 = time.perf_counter()
    lat, st = bench.serve_trial(pipe, N, pos, bufs, warm, meas, max_batch=max_batch,
                                graphs=graph)
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
    if use_graph:
        # every step a replay of a bucket-sized graph: pieces of 4, then 2, the
        # last padded with the spare slots N, N + 1
        assert all(len(sl) in (4, 2) for _, sl in pipe.calls)
        assert st["steps"] <= len(pipe.calls)
        assert sum(g[0].replays for g in graph.g.values()) - replays0 == len(pipe.calls)
        padded = [sl for _, sl in pipe.calls if N in sl or N + 1 in sl]
        assert padded, "odd batches should have been padded"
        for sl in padded:
            real = [x for x in sl if x < N]
            assert sl[len(real):] == [N, N + 1][:len(sl) - len(real)]
        assert pipe.pool.flushes > 0   # (streams ended in the last iteration wait for a next step)
    else:
        assert st["steps"] == len(pipe.calls)
        full = [sl for c, sl in pipe.calls if c == 2 and len(sl) == max_batch]
        assert full, "the trial should have made full later-chunk batches"


@pytest.mark.parametrize("B", [1, 127, 128, 129, 300, 1024, 1500, 2047, 2048])
def test_step_graph_pieces_cover_the_batch_with_little_padding(B):
    """StepGraphs.pieces: bucket-sized replays, largest first, covering the
    batch's rows once; only the last is padded, to the smallest bucket."""
    g = bench.StepGraphs.__new__(bench.StepGraphs)
    g.sizes = sorted(bench.STEP_BUCKETS, reverse=True)
    pieces = g.pieces(B)
    assert sum(r for r, _ in pieces) == B
    assert all(r == Bg for r, Bg in pieces[:-1])
    r, Bg = pieces[-1]
    assert r == Bg or (Bg == min(bench.STEP_BUCKETS) and r < Bg)
    assert [Bg for _, Bg in pieces] == sorted((Bg for _, Bg in pieces), reverse=True)
    assert Bg - r < min(bench.STEP_BUCKETS)   # padding fits the spare slots
