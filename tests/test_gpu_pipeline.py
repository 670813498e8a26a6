"""The features -> tokens streaming step (parakeet_b200.engine.pipeline) on the
GPU: a batch of streams stepped together gives each stream the same tokens as
stepping it alone (slot isolation of the three per-slot states: mel cache,
K/V pages + conv cache, prediction state), in fp32, over a first chunk and
later chunks; and one steady-state step replays as a CUDA graph with the same
result.  The same for the audio -> tokens step (sample history as a fourth
per-slot state), and for the overlapped runner that decodes chunk k on a second
stream under chunk k+1's encoder."""
import numpy as np
import pytest
import torch

from parakeet_b200.engine import OverlappedStreamingRunner, StreamingPipeline
from parakeet_b200.modules import ConformerEncoder, Joiner, Predictor
from parakeet_b200.weights import (random_decoder_state_dict, random_encoder_layers,
                                   random_pre_encode_state_dict)

pytestmark = pytest.mark.gpu
D, LAYERS, HEADS, V = 512, 2, 8, 1026


def make(num_slots, **kw):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    enc = ConformerEncoder(feat_in=128, hidden_size=D, ff_expansion_factor=4, num_layers=LAYERS,
                           num_heads=HEADS, subsampling_factor=8, pos_emb_max_len=5000,
                           conv_kernel_size=9, att_context_size=(70, 1),
                           subsampling_conv_channels=256, use_bias=False)
    sd = {**random_encoder_layers(3, LAYERS, D, HEADS),
          **{f"pre_encode.{k}": v for k, v in random_pre_encode_state_dict(4, 128, 256, D).items()}}
    enc.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
    pre = enc.pre_encode
    sd = random_decoder_state_dict(5, D, 640, 640, V, 1, blank_bias=2.3)
    pred, join = Predictor(640, 640, 1, V), Joiner(D, 640, 640, num_classes=V)
    pred.load_state_dict({k[10:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("predictor.")})
    join.load_state_dict({k[7:]: torch.from_numpy(v) for k, v in sd.items()
                          if k.startswith("joiner.")})
    mods = [m.to("cuda", torch.float32).eval() for m in (enc, pre, pred, join)]
    return StreamingPipeline(*mods, blank_id=V, num_slots=num_slots, **kw)


def feats(step, i):
    g = torch.Generator().manual_seed(1000 * step + i)
    return torch.randn(1, 128, 9 if step == 0 else 16, generator=g)


def run(streams, steps, pipe, slot_of):
    out = {}
    with torch.inference_mode():
        for step in range(steps):
            f = torch.cat([feats(step, i) for i in streams]).cuda()
            slots = torch.tensor([slot_of[i] for i in streams], dtype=torch.int32, device="cuda")
            tok, cnt = pipe.step(f, slots, first=step == 0)
            tok, cnt = tok.cpu(), cnt.cpu()
            for r, i in enumerate(streams):
                out[(step, i)] = [int(x) for t in range(tok.shape[1])
                                  for x in tok[r, t, : int(cnt[r, t])]]
    return out


def test_batched_step_equals_streams_alone():
    streams, steps = [0, 1, 2], 5
    pipe = make(4)
    pipe.start_streams([3, 1, 0])
    together = run(streams, steps, pipe, {0: 3, 1: 1, 2: 0})
    for i in streams:
        alone_pipe = make(1)
        alone_pipe.start_streams([0])
        alone = run([i], steps, alone_pipe, {i: 0})
        for step in range(steps):
            assert together[(step, i)] == alone[(step, i)], (step, i)
    assert sum(len(v) for v in together.values()) > 0
    assert pipe.pool.read_error() == 0


def test_steady_step_replays_as_cuda_graph():
    pipe, ref_pipe = make(2), make(2)
    pipe.start_streams([0, 1])
    ref_pipe.start_streams([0, 1])
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    with torch.inference_mode():
        pipe.step(torch.cat([feats(0, 0), feats(0, 1)]).cuda(), slots, first=True)
        f = torch.cat([feats(1, 0), feats(1, 1)]).cuda()
        ref_pipe.step(torch.cat([feats(0, 0), feats(0, 1)]).cuda(), slots, first=True)
        want = ref_pipe.step(f, slots, first=False)
        g = torch.cuda.CUDAGraph()
        static_f = f.clone()
        with torch.cuda.graph(g):
            tok, cnt = pipe.step(static_f, slots, first=False)
    # the capture ran no kernels: replaying it now performs this step
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(tok, want[0]) and torch.equal(cnt, want[1])


SMALL_FIRST, SMALL_NEXT = 9 * 160, 16 * 160     # samples per chunk, lookahead 1


def audio(step, i):
    rng = np.random.default_rng(7000 + 100 * i + step)
    n = SMALL_FIRST if step == 0 else SMALL_NEXT
    t = np.arange(n) / 16000.0
    f = rng.uniform(100, 4000, 3)
    x = sum(np.sin(2 * np.pi * fk * t + rng.uniform(0, 6.3)) for fk in f) / 3
    x = x + 0.1 * rng.standard_normal(n)
    return torch.from_numpy((0.4 * x).astype(np.float32))[None]


def run_audio(streams, steps, pipe, slot_of):
    out = {}
    with torch.inference_mode():
        for step in range(steps):
            x = torch.cat([audio(step, i) for i in streams]).cuda()
            slots = torch.tensor([slot_of[i] for i in streams], dtype=torch.int32, device="cuda")
            tok, cnt = pipe.step_audio(x, slots, push=step)
            tok, cnt = tok.cpu(), cnt.cpu()
            for r, i in enumerate(streams):
                out[(step, i)] = [int(x) for t in range(tok.shape[1])
                                  for x in tok[r, t, : int(cnt[r, t])]]
    return out


def test_audio_step_is_features_then_step():
    """step_audio = the extractor's push_batch followed by step."""
    a, b = make(3), make(3)
    slots = [2, 0]
    a.start_streams(slots)
    b.start_streams(slots)
    sl = torch.tensor(slots, dtype=torch.int32, device="cuda")
    with torch.inference_mode():
        for step in range(4):
            x = torch.cat([audio(step, i) for i in range(2)]).cuda()
            ta, ca = a.step_audio(x, sl, push=step)
            f, counts = b.fe.push_batch(x, slots, first=step == 0)
            assert list(counts) == [8 if step == 0 else 16] * 2
            # the second window takes the 8 frames the first one left in the cache
            tb, cb = b.step(f, sl, first=step == 0, prefix=8 if step == 1 else None)
            assert torch.equal(ta, tb) and torch.equal(ca, cb), step
    assert a.fe.error_bits() == 0


def test_audio_batched_step_equals_streams_alone():
    streams, steps = [0, 1, 2], 5
    kw = dict(feature_kw=dict(dither=0.0))
    pipe = make(4, **kw)
    pipe.start_streams([3, 1, 0])
    together = run_audio(streams, steps, pipe, {0: 3, 1: 1, 2: 0})
    for i in streams:
        alone_pipe = make(1, **kw)
        alone_pipe.start_streams([0])
        alone = run_audio([i], steps, alone_pipe, {i: 0})
        for step in range(steps):
            assert together[(step, i)] == alone[(step, i)], (step, i)
    assert sum(len(v) for v in together.values()) > 0


def test_audio_steady_step_replays_as_cuda_graph():
    pipe, ref_pipe = make(2), make(2)
    pipe.start_streams([0, 1])
    ref_pipe.start_streams([0, 1])
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    with torch.inference_mode():
        for push in range(2):
            x = torch.cat([audio(push, 0), audio(push, 1)]).cuda()
            pipe.step_audio(x, slots, push)
            ref_pipe.step_audio(x, slots, push)
        x2 = torch.cat([audio(2, 0), audio(2, 1)]).cuda()
        want = ref_pipe.step_audio(x2, slots, 2)
        static_x = x2.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            tok, cnt = pipe.step_audio(static_x, slots, 2)
    # the capture ran no kernels: replaying it now performs push 2
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(tok, want[0]) and torch.equal(cnt, want[1])


def test_overlapped_runner_equals_sequential_steps():
    """OverlappedStreamingRunner: chunk k's decode on the decode stream under
    chunk k+1's features + encoder gives every chunk the tokens of plain
    sequential step_audio calls; outputs of step k are read only after its
    event, and before the step two calls later reuses its buffers."""
    pipe, ref_pipe = make(3), make(3)
    slots_l = [2, 0, 1]
    pipe.start_streams(slots_l)
    ref_pipe.start_streams(slots_l)
    slots = torch.tensor(slots_l, dtype=torch.int32, device="cuda")
    n = 7
    xs = [torch.cat([audio(p, i) for i in range(3)]).cuda() for p in range(2 + n)]
    with torch.inference_mode():
        for push in range(2):
            pipe.step_audio(xs[push], slots, push)
            ref_pipe.step_audio(xs[push], slots, push)
        want = [ref_pipe.step_audio(xs[2 + k], slots, 2) for k in range(n)]
        want = [(t.clone(), c.clone()) for t, c in want]
        runner = OverlappedStreamingRunner(pipe, slots, SMALL_NEXT)
        main = torch.cuda.current_stream()
        got, prev = [], None
        for k in range(n):
            cur = runner.step(xs[2 + k])
            if prev is not None:
                main.wait_event(prev[2])
                got.append((prev[0].clone(), prev[1].clone()))
            prev = cur
        runner.drain()
        got.append((prev[0].clone(), prev[1].clone()))
        torch.cuda.synchronize()
    for k in range(n):
        assert torch.equal(got[k][0], want[k][0]) and torch.equal(got[k][1], want[k][1]), k
    assert sum(int(c.sum()) for _, c in want) > 0
    assert pipe.pool.read_error() == 0 and pipe.fe.error_bits() == 0


def test_captured_step_survives_other_batch_sizes():
    """A step captured as a CUDA graph keeps working after the pipeline has run
    many other batch sizes eagerly: the feature buffers the graph reads must not
    be evicted (and their memory reused) by the cache of recent batch sizes."""
    pipe, ref_pipe = make(24), make(24)
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    pipe.start_streams([0, 1])
    ref_pipe.start_streams([0, 1])
    with torch.inference_mode():
        for push in range(2):
            x = torch.cat([audio(push, 0), audio(push, 1)]).cuda()
            pipe.step_audio(x, slots, push)
            ref_pipe.step_audio(x, slots, push)
        x2 = torch.cat([audio(2, 0), audio(2, 1)]).cuda()
        static_x = x2.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            tok, cnt = pipe.step_audio(static_x, slots, 2)
        # first chunks of other streams at 20 batch sizes: more than the cache holds
        for rep in range(2):
            for B in range(1, 21):
                other = torch.arange(2, 2 + B, dtype=torch.int32, device="cuda")
                pipe.start_streams(other)
                xb = torch.cat([audio(0, 10 + i) for i in range(B)]).cuda()
                pipe.step_audio(xb, other, 0)
        want = ref_pipe.step_audio(x2, slots, 2)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(tok, want[0]) and torch.equal(cnt, want[1])
    assert pipe.fe.error_bits() == 0 and pipe.pool.read_error() == 0


def test_graphs_of_two_push_indices_share_buffers_in_any_replay_order():
    """Steps of push 1 and of push 2 captured at one batch size share the
    feature buffers (same samples, not first); replaying the push-2 graph
    before the push-1 graph ever ran still counts the right samples."""
    pipe, ref_pipe = make(3), make(3)
    sl = [0, 1, 2]
    slots = torch.tensor(sl, dtype=torch.int32, device="cuda")
    pipe.start_streams(sl)
    ref_pipe.start_streams(sl)
    with torch.inference_mode():
        x0 = torch.cat([audio(0, i) for i in sl]).cuda()
        x1 = torch.cat([audio(1, i) for i in sl]).cuda()
        x2 = torch.cat([audio(2, i) for i in sl]).cuda()
        pipe.step_audio(x0, slots, 0)
        for p, x in enumerate((x0, x1)):
            ref_pipe.step_audio(x, slots, p)
        want = ref_pipe.step_audio(x2, slots, 2)
        gx1, gx2 = x1.clone(), x2.clone()
        g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            pipe.step_audio(gx1, slots, 1)
        with torch.cuda.graph(g2):
            tok, cnt = pipe.step_audio(gx2, slots, 2)
        # push 1 eagerly at other batch sizes (g1 never replays)
        pipe.step_audio(x1[:2], slots[:2], 1)
        pipe.step_audio(x1[2:], slots[2:], 1)
    g2.replay()
    torch.cuda.synchronize()
    assert torch.equal(tok, want[0]) and torch.equal(cnt, want[1])
    assert pipe.fe.error_bits() == 0 and pipe.pool.read_error() == 0
