"""GPU streaming log-mel features (pk_features_push through the C-ABI)
against the reference extractor's own outputs (tests/golden/features.npz)
and the float64 oracle (oracle/features.py)."""
import os
import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden_features import (FULL, LARGE_FIRST, LARGE_NEXT, SMALL_FIRST,  # noqa: E402
                                  SMALL_NEXT, STREAMS)
from oracle.features import FeatureStream, LogMel, synth_audio  # noqa: E402

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(HERE, "golden", "features.npz"))
# log-mel, absolute: fp32 FFT on the GPU vs the reference (fp32) / oracle (fp64)
TOL = 2e-3


def extractor(**kw):
    from parakeet_b200.modules import FeatureExtractor
    kw.setdefault("dither", 0.0)
    return FeatureExtractor(device="cuda", **kw)


def sequence(slot):
    return SimpleNamespace(encoder_state=slot, _fe_samples=np.empty((0,), np.float32),
                           _fe_emitted_frames=0, _fe_sample_offset=0)


@pytest.mark.parametrize("name", sorted(STREAMS))
def test_push_drop_in_matches_reference(name):
    """The reference's push(samples, state, final) call sequence, one stream."""
    seed, pushes = STREAMS[name]
    fe = extractor(num_slots=4)
    audio = synth_audio(seed, sum(n for n, _ in pushes))
    st, pos, frames, counts = sequence(2), 0, [], []
    for n, final in pushes:
        f = fe.push(audio[pos:pos + n], st, final=final)
        pos += n
        counts.append(0 if f is None else f.shape[-1])
        if f is not None:
            assert f.shape[:2] == (1, 128)
            frames.append(f[0].float().cpu().numpy())
    assert counts == list(GOLD[f"{name}_counts"])
    got = np.concatenate(frames, 1) if frames else np.zeros((128, 0))
    ref = GOLD[f"{name}_feats"]
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= TOL
    assert fe.error_bits() == 0


def test_call_matches_reference():
    fe = extractor()
    for name, (seed, n) in FULL.items():
        got = fe(synth_audio(seed, n))[0].cpu().numpy()
        ref = GOLD[f"{name}_feats"]
        assert got.shape == ref.shape
        assert np.abs(got - ref).max() <= TOL
    # a second utterance on the same extractor starts afresh
    got = fe(synth_audio(FULL["full_3000"][0], 3000))[0].cpu().numpy()
    assert np.abs(got - GOLD["full_3000_feats"]).max() <= TOL


def run_batched(fe, streams, schedule, rng=None):
    """schedule: list of steps, each {row: (n, final)}; every row's first push
    is its first.  Returns per-row concatenated GPU frames and oracle frames."""
    mel = LogMel()
    total = {r: sum(step[r][0] for step in schedule if r in step) for r in streams}
    audio = {r: synth_audio(1000 + r, total[r]) for r in streams}
    pos = {r: 0 for r in streams}
    oracle = {r: FeatureStream(mel) for r in streams}
    got = {r: [] for r in streams}
    want = {r: [] for r in streams}
    started = set()
    for step in schedule:
        rows = sorted(step)
        nmax = max(step[r][0] for r in rows)
        x = np.zeros((len(rows), nmax), np.float32)
        ns, firsts, finals = [], [], []
        for i, r in enumerate(rows):
            n, final = step[r]
            x[i, :n] = audio[r][pos[r]:pos[r] + n]
            f = oracle[r].push(audio[r][pos[r]:pos[r] + n], final)
            if f is not None:
                want[r].append(f)
            pos[r] += n
            ns.append(n)
            firsts.append(r not in started)
            finals.append(final)
            started.add(r)
        out, counts = fe.push_batch(x, [streams[r] for r in rows], first=firsts, final=finals,
                                    num_samples=ns)
        out = out.float().cpu().numpy()
        for i, r in enumerate(rows):
            got[r].append(out[i, :, :counts[i]])
            assert np.all(out[i, :, counts[i]:] == fe.pad_value)
    cat = lambda fs: np.concatenate(fs, 1) if fs else np.zeros((128, 0))  # noqa: E731
    return {r: cat(got[r]) for r in streams}, {r: cat(want[r]) for r in streams}


def check(got, want, tol=TOL):
    for r in want:
        assert got[r].shape == want[r].shape, r
        if want[r].size:
            assert np.abs(got[r] - want[r]).max() <= tol, r


def test_batched_small_chunks_with_joins_and_finals():
    fe = extractor(num_slots=32)
    streams = {r: (7 * r + 3) % 32 for r in range(12)}
    sched = []
    for s in range(6):
        step = {}
        for r in range(12):
            start = r % 3
            if s < start:
                continue
            k = s - start
            if r == 5 and k == 3:
                step[r] = (900, True)          # final, shorter chunk
            elif r == 5 and k > 3:
                continue
            else:
                step[r] = (SMALL_FIRST if k == 0 else SMALL_NEXT, False)
        sched.append(step)
    got, want = run_batched(fe, streams, sched)
    check(got, want)
    assert fe.error_bits() == 0


def test_batched_ragged_counts():
    """Different sample counts in one push, including empty and tiny ones."""
    fe = extractor(num_slots=8)
    streams = {r: r for r in range(6)}
    rng = np.random.default_rng(5)
    sched = []
    for s in range(7):
        step = {}
        for r in range(6):
            n = int(rng.choice([0, 3, 37, 160, 255, 256, 257, 800, 2560, 4111]))
            step[r] = (n, s == 6 and r % 2 == 0)
        sched.append(step)
    got, want = run_batched(fe, streams, sched)
    check(got, want)
    assert fe.error_bits() == 0


def test_batched_large_chunks_many_streams():
    """Large-model chunks (16800 then 17920 samples) for 96 streams: the launch
    takes 32 frames per CTA here."""
    fe = extractor(num_slots=128)
    streams = {r: 127 - r for r in range(96)}
    sched = [{r: (LARGE_FIRST, False) for r in range(96)},
             {r: (LARGE_NEXT, False) for r in range(96)},
             {r: (2000, True) for r in range(0, 96, 5)}]
    got, want = run_batched(fe, streams, sched)
    check(got, want)
    assert fe.error_bits() == 0


def test_bf16_output_is_rounded_fp32():
    a = extractor(num_slots=4)
    b = extractor(num_slots=4, out_dtype=torch.bfloat16)
    x = np.stack([synth_audio(9 + i, SMALL_FIRST) for i in range(3)])
    fa, ca = a.push_batch(x, [0, 1, 2], first=True)
    fb, cb = b.push_batch(x, [0, 1, 2], first=True)
    assert fb.dtype == torch.bfloat16 and list(ca) == list(cb)
    ref = fa.float()
    err = (fb.float() - ref).abs()
    assert bool((err <= ref.abs() * 2 ** -8 + 1e-6).all())


def test_dither_distribution_and_reproducibility():
    """Silence with dither: per-bin mean log-mel matches the oracle's (numpy
    Gaussian dither) within sampling error; one seed reproduces itself.  The
    dither is 1e-3 here so that the noise power stands well above the log
    guard (at the default 1e-5 every bin reads log(guard + tiny))."""
    n = 160 * 400
    x = np.zeros((1, n), np.float32)
    outs = []
    for seed in (1, 1, 2):
        fe = extractor(dither=1e-3, seed=seed)
        f, _ = fe.push_batch(x, [0], first=True, final=True)
        outs.append(f[0].cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert not np.array_equal(outs[0], outs[2])
    want = LogMel().compute(x[0], dither=1e-3, rng=np.random.default_rng(0))
    got = outs[0]
    inner = slice(3, -3)                                  # frames away from the zero padding
    assert got.shape == want.shape
    dm = got[:, inner].mean(1) - want[:, inner].mean(1)
    # per bin: ~395 overlapping frames of a log-chi-square variable
    assert np.abs(dm).max() < 0.75
    assert abs(dm.mean()) < 0.05


def test_device_errors_do_not_fault():
    """A bad slot or count sets a bit in the error word; the row's output is
    padding and its count 0; the other rows are unaffected."""
    from parakeet_b200._lib import PK_DEV_BAD_COUNT, PK_DEV_BAD_SLOT
    fe = extractor(num_slots=4)
    dev = torch.device("cuda")
    x = torch.from_numpy(np.stack([synth_audio(3, 1600)] * 3)).to(dev)
    ns = torch.tensor([1600, 1600, 1600], dtype=torch.int32, device=dev)
    flags = torch.ones(3, dtype=torch.int32, device=dev)
    slots = torch.tensor([0, 99, 1], dtype=torch.int32, device=dev)
    out = torch.empty(3, 128, 9, device=dev)
    nf = torch.empty(3, dtype=torch.int32, device=dev)
    fe.launch(x, ns, flags, slots, out, 9, nf)
    torch.cuda.synchronize()
    assert fe.error_bits() & PK_DEV_BAD_SLOT
    assert nf.tolist() == [9, 0, 9]          # (1600 - 256) // 160 + 1
    assert bool((out[1] == fe.pad_value).all())
    assert torch.equal(out[0], out[2])
    fe.error.zero_()
    ns2 = torch.tensor([1600, 5000, 1600], dtype=torch.int32, device=dev)
    slots2 = torch.tensor([2, 3, 0], dtype=torch.int32, device=dev)
    fe.launch(x, ns2, flags, slots2, out, 9, nf)
    torch.cuda.synchronize()
    assert fe.error_bits() == PK_DEV_BAD_COUNT
    assert nf.tolist() == [9, 0, 9]          # (1600 - 256) // 160 + 1
    fe.error.zero_()
    # more frames than max_frames: the first max_frames are kept
    out4 = torch.empty(3, 128, 4, device=dev)
    slots3 = torch.tensor([1, 2, 3], dtype=torch.int32, device=dev)
    fe.launch(x, ns, flags, slots3, out4, 4, nf)
    torch.cuda.synchronize()
    assert fe.error_bits() == PK_DEV_BAD_COUNT
    assert nf.tolist() == [4, 4, 4]
    assert torch.equal(out4[0], out[0, :, :4])


def test_graph_replay_matches_eager():
    """Steady-state pushes captured once in a CUDA graph and replayed with new
    samples give the eager extractor's frames."""
    B, dev = 16, torch.device("cuda")
    eager, graphed = extractor(num_slots=B), extractor(num_slots=B)
    audio = np.stack([synth_audio(50 + i, SMALL_FIRST + 6 * SMALL_NEXT) for i in range(B)])
    slots = list(range(B))
    e0, _ = eager.push_batch(audio[:, :SMALL_FIRST], slots, first=True)
    g0, _ = graphed.push_batch(audio[:, :SMALL_FIRST], slots, first=True)
    assert torch.equal(e0, g0)
    x = torch.zeros(B, SMALL_NEXT, device=dev)
    ns = torch.full((B,), SMALL_NEXT, dtype=torch.int32, device=dev)
    flags = torch.zeros(B, dtype=torch.int32, device=dev)
    sl = torch.arange(B, dtype=torch.int32, device=dev)
    out = torch.empty(B, 128, 16, device=dev)
    nf = torch.empty(B, dtype=torch.int32, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        graphed.launch(x, ns, flags, sl, out, 16, nf)
    torch.cuda.current_stream().wait_stream(s)
    for k in range(6):
        chunk = audio[:, SMALL_FIRST + k * SMALL_NEXT:SMALL_FIRST + (k + 1) * SMALL_NEXT]
        want, counts = eager.push_batch(chunk, slots)
        x.copy_(torch.from_numpy(chunk))
        g.replay()
        torch.cuda.synchronize()
        assert list(counts) == [16] * B and nf.tolist() == [16] * B
        assert torch.equal(out, want)
    del g
