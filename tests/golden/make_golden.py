"""Generate the golden vectors in this directory by running the reference.

Runs odunola499/parakeet-streaming's own modules (imported from a source
checkout given by ``--reference``) on seeded inputs and saves their outputs
as small ``.npz`` fixtures.  The fixtures are committed; the GPU box never
needs the reference.  Three shims make the reference importable offline:

* ``librosa`` is not installed: a stub ``librosa.filters.mel`` returns
  torchaudio's slaney mel bank (only the feature extractor uses it, which is
  off the hot path);
* weights come from ``parakeet_b200.weights`` (seeded numpy) and are loaded
  with ``load_state_dict``, because HF downloads are impossible offline;
* sequences are plain objects with an ``encoder_state`` slot id, which is all
  ``Scheduler.pack_states`` reads (parakeet/engine/scheduler.py:136).

Usage:  python tests/golden/make_golden.py --reference <path to reference>
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
from parakeet_b200.weights import random_encoder_layers, seeded_normal  # noqa: E402

sys.path.insert(0, os.path.join(REPO, "baseline"))
from harness import install_librosa_stub  # noqa: E402,F401  (also used by the other generators)


# Streams used by the encoder fixtures: (name, acquire step, release step or
# None, step whose chunk is short).  A stream runs in steps acquire <= s < release
# and is released at the start of step ``release``; a short chunk (length 1 < T)
# is only ever that stream's last step, like a final chunk.
SMALL_SCHEDULE = dict(att=(70, 1), dim=512, heads=8, layers=2, steps=40, pool=4,
                      seed=11, events=[("a", 0, None, None), ("b", 0, 21, None),
                                       ("c", 6, None, None), ("d", 22, None, 39),
                                       ("e", 25, None, None)],
                      keep_steps=[0, 1, 2, 17, 34, 35, 36, 38, 39])
LARGE_SCHEDULE = dict(att=(70, 13), dim=1024, heads=8, layers=1, steps=8, pool=3,
                      seed=12, events=[("a", 0, None, None), ("b", 2, None, None)],
                      keep_steps=[1, 6, 7])


# The same schedules through the whole stack (17 layers small, 24 large:
# parakeet/config.py:7,27).  Their fixtures also hold how far the reference's
# own bf16 run lands from its fp32 run at each kept step: bf16 rounding alone
# moves a 17-24 layer stack of random weights by 2-3 % rel-L2, which is the
# scale a bf16 implementation is held to at full depth.
SMALL_FULL = dict(SMALL_SCHEDULE, layers=17)
LARGE_FULL = dict(LARGE_SCHEDULE, layers=24)


# 256 streams arriving as a Poisson process (mean 20 per second)
# with lengths uniform in 2-120 s, one 160 ms chunk per stream per step; the
# page pool holds 60 % of the full demand (256 streams x 6 pages), which admits
# floor(0.6 * 256) = 153 streams at once; the others wait in arrival order.
CHURN = dict(streams=256, rate=20.0, min_s=2.0, max_s=120.0, period=0.16, cap=0.6,
             pages_per_stream=6, seed=41)


def churn_schedule(cfg=CHURN):
    """(arrival step, chunks) per stream, seeded."""
    rng = np.random.default_rng(cfg["seed"])
    t = np.cumsum(rng.exponential(1.0 / cfg["rate"], cfg["streams"]))
    secs = rng.uniform(cfg["min_s"], cfg["max_s"], cfg["streams"])
    return (np.floor(t / cfg["period"]).astype(np.int64),
            np.maximum(1, np.round(secs / cfg["period"])).astype(np.int64))


def churn_replay(acquire, release, cfg=CHURN, on_step=None):
    """The engine's admission loop over ``churn_schedule``: each step, the
    streams that sent their last chunk in the previous step are released (in
    admission order), the step's arrivals join the waiting queue, waiting
    streams are admitted in arrival order while ``acquire()`` gives a slot,
    and every live stream sends one chunk (its last one of length 1, a short
    final chunk).  ``on_step(step, slots, lengths, released)`` sees each step.
    Returns the slot operations [(step, op 0 = acquire / 1 = release, stream,
    slot)]."""
    from collections import deque
    arrive, chunks = churn_schedule(cfg)
    waiting, live, ops = deque(), {}, []          # live: stream -> [slot, chunks left]
    step, nxt = 0, 0
    while nxt < len(arrive) or waiting or live:
        released = []
        for sid in [s for s, (_, left) in live.items() if left == 0]:
            slot = live.pop(sid)[0]
            release(slot)
            ops.append((step, 1, sid, slot))
            released.append(slot)
        while nxt < len(arrive) and arrive[nxt] <= step:
            waiting.append(nxt)
            nxt += 1
        while waiting:
            slot = acquire()
            if slot is None:
                break
            sid = waiting.popleft()
            live[sid] = [slot, int(chunks[sid])]
            ops.append((step, 0, sid, slot))
        slots, lengths = [], []
        for sid, rec in live.items():
            slots.append(rec[0])
            lengths.append(1 if rec[1] == 1 else None)
            rec[1] -= 1
        if on_step is not None:
            on_step(step, slots, lengths, released)
        step += 1
    return ops


def churn_fixture():
    """The reference Scheduler's slot ids (scheduler.py:86-104, a pool of the
    153 streams the capped page pool admits) under configs[4]'s churn."""
    from parakeet.engine.scheduler import Scheduler
    from parakeet.modules.cache import ModelCache, StreamingState

    class TinyEncoder:
        def init_streaming_state(self, batch_size, device, dtype):
            return StreamingState(ModelCache(1, (70, 1), 4, 9, batch_size, device, dtype),
                                  torch.zeros(batch_size, dtype=torch.int64),
                                  torch.zeros(batch_size, dtype=torch.int64))

    sched = Scheduler()
    n = int(CHURN["cap"] * CHURN["streams"])
    sched.init_state_pool(TinyEncoder(), torch.device("cpu"), torch.float32, n)
    live = [0, 0]

    def count(step, slots, lengths, released):
        live[0] = max(live[0], len(slots))
        live[1] = step + 1

    ops = churn_replay(sched.acquire_state_slot, sched.release_state_slot, on_step=count)
    return {"ops": np.array(ops, np.int64), "max_live": np.array(live[0]),
            "steps": np.array(live[1])}


def encoder_stream_inputs(seed, step, batch, T, dim):
    """Chunk input of one step: N(0,1) [batch, T, dim] from seed*1000+step."""
    return seeded_normal(seed * 1000 + step, (batch, T, dim))


def schedule_batches(cfg):
    """Per step: [(stream name, length)] in acquisition order, which is the
    order ``Scheduler.active`` (a deque, scheduler.py:24) hands them out."""
    T = cfg["att"][1] + 1
    steps = []
    for s in range(cfg["steps"]):
        live = [e for e in cfg["events"] if e[1] <= s and (e[2] is None or s < e[2])]
        steps.append([(e[0], 1 if e[3] == s else T) for e in live])
    return steps


def run_encoder_fixture(ref, cfg, dtype=torch.float32):
    from parakeet.modules import ConformerEncoder
    from parakeet.engine.scheduler import Scheduler

    left, right = cfg["att"]
    T = right + 1
    torch.manual_seed(0)
    enc = ConformerEncoder(feat_in=128, hidden_size=cfg["dim"], ff_expansion_factor=4,
                           num_layers=cfg["layers"], num_heads=cfg["heads"],
                           subsampling_factor=8, pos_emb_max_len=5000,
                           conv_kernel_size=9, att_context_size=cfg["att"],
                           subsampling_conv_channels=256, use_bias=False)
    sd = random_encoder_layers(cfg["seed"], cfg["layers"], cfg["dim"], cfg["heads"])
    missing, unexpected = enc.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()},
                                              strict=False)
    assert not unexpected and all(not k.startswith("layers.") for k in missing), missing
    enc = enc.to(dtype).eval()
    sched = Scheduler(max_active=cfg["pool"])
    sched.init_state_pool(enc, torch.device("cpu"), dtype, cfg["pool"])
    slot_of, acquired, released = {}, [], []
    outs, lens, slots = {}, {}, {}
    batches = schedule_batches(cfg)
    for s, batch in enumerate(batches):
        for name, acq, rel, _ in cfg["events"]:
            if rel == s:
                sched.release_state_slot(slot_of[name])
                released.append((s, slot_of[name]))
        for name, acq, rel, _ in cfg["events"]:
            if acq == s:
                slot_of[name] = sched.acquire_state_slot()
                acquired.append((s, slot_of[name]))
        seqs = [SimpleNamespace(encoder_state=slot_of[n]) for n, _ in batch]
        x = torch.from_numpy(encoder_stream_inputs(cfg["seed"], s, len(batch), T, cfg["dim"]))
        x = x.to(dtype)
        length = torch.tensor([n for _, n in batch], dtype=torch.int64)
        st, idx = sched.pack_states(seqs)
        with torch.inference_mode():
            y, st = enc(x, st, length=length, bypass_pre_encode=True)
        sched.unpack_states(st, idx)
        if s in cfg["keep_steps"]:
            outs[s] = y.float().numpy()
            lens[s] = length.numpy()
            slots[s] = idx.numpy()
    fx = {"keep_steps": np.array(cfg["keep_steps"]),
          "acquired": np.array(acquired, np.int64),
          "released": np.array(released, np.int64).reshape(-1, 2),
          "final_processed": sched._pool_state.processed_frames.numpy(),
          "final_cache_len": sched._pool_state.cache_lengths.numpy(),
          "final_conv_l0": sched._pool_state.cache.conv[:, 0].float().numpy(),
          "final_k_l0_last": sched._pool_state.cache.attn_k[:, 0, -T:].float().numpy()}
    for s in cfg["keep_steps"]:
        fx[f"out_{s}"] = outs[s]
        fx[f"len_{s}"] = lens[s]
        fx[f"slots_{s}"] = slots[s]
    return fx


def cache_window_fixture(att, dim, steps, batch, layers, seed):
    from parakeet.modules.cache import ModelCache

    T = att[1] + 1
    cache = ModelCache(layers, att, dim, 9, batch_size=batch, dtype=torch.float32)
    rng = np.random.default_rng(seed)
    keys = rng.standard_normal((steps, layers, batch, T, dim)).astype(np.float32)
    vals = rng.standard_normal((steps, layers, batch, T, dim)).astype(np.float32)
    wk = np.zeros((steps, layers, batch, att[0] + T, dim), np.float32)
    wv = np.zeros_like(wk)
    for s in range(steps):
        for l in range(layers):
            k, v = cache.update_attn_cache(l, torch.from_numpy(keys[s, l]),
                                           torch.from_numpy(vals[s, l]))
            wk[s, l], wv[s, l] = k.numpy(), v.numpy()
    return {"keys": keys, "values": vals, "win_k": wk, "win_v": wv}


def masks_fixture():
    from parakeet.modules.encoder import ConformerEncoder

    out = {}
    rng = np.random.default_rng(5)
    for tag, att in (("small", (70, 1)), ("large", (70, 13))):
        T = att[1] + 1
        cl, pf, ln = [], [], []
        # aligned streams at every fill level, unaligned histories, short chunks
        for proc in (0, 2, 14, 28, 68, 70, 72, 140, 1000):
            cl.append(min(proc, 70)); pf.append(proc); ln.append(T)
        for _ in range(12):
            proc = int(rng.integers(0, 300))
            cl.append(int(rng.integers(0, min(proc, 70) + 1))); pf.append(proc)
            ln.append(int(rng.integers(1, T + 1)))
        me = SimpleNamespace(att_context_size=att)
        pad, mask = ConformerEncoder._create_streaming_masks(
            me, T, torch.tensor(cl), torch.tensor(pf), torch.device("cpu"), torch.tensor(ln))
        out[f"{tag}_cache_len"] = np.array(cl)
        out[f"{tag}_processed"] = np.array(pf)
        out[f"{tag}_lengths"] = np.array(ln)
        out[f"{tag}_pad"] = pad.numpy()
        out[f"{tag}_att"] = mask.numpy()
    return out


def scheduler_fixture():
    """Slot ids returned by the reference Scheduler under seeded churn."""
    from parakeet.engine.scheduler import Scheduler
    from parakeet.modules.cache import ModelCache, StreamingState

    class TinyEncoder:
        def init_streaming_state(self, batch_size, device, dtype):
            return StreamingState(ModelCache(1, (70, 1), 4, 9, batch_size, device, dtype),
                                  torch.zeros(batch_size, dtype=torch.int64),
                                  torch.zeros(batch_size, dtype=torch.int64))

    sched = Scheduler()
    sched.init_state_pool(TinyEncoder(), torch.device("cpu"), torch.float32, 8)
    rng = np.random.default_rng(9)
    held, ops = [], []
    for _ in range(200):
        if held and (rng.random() < 0.45 or len(held) == 8 and rng.random() < 0.5):
            slot = held.pop(int(rng.integers(len(held))))
            sched.release_state_slot(slot)
            ops.append((1, slot))
        else:
            slot = sched.acquire_state_slot()
            ops.append((0, -1 if slot is None else slot))
            if slot is not None:
                held.append(slot)
    return {"ops": np.array(ops, np.int64)}


def admission_fixture():
    """The reference Scheduler's admission queue (scheduler.py:35-66) under
    seeded add / admit_ready / release calls, max_active 3: per call, the
    sequences admitted, the running sequences in order and every sequence's
    status.  Sequences are plain objects holding a status of the reference's
    ``SequenceStatus`` (what ``Sequence.__init__`` sets, sequence.py:33)."""
    import json

    from parakeet.engine.scheduler import Scheduler
    from parakeet.engine.sequence import SequenceStatus

    sched = Scheduler(max_active=3)
    rng = np.random.default_rng(13)
    seqs, calls = [], []
    for _ in range(300):
        u = rng.random()
        if u < 0.4 or not seqs:
            seq = SimpleNamespace(status=SequenceStatus.WAITING, name=len(seqs))
            seqs.append(seq)
            sched.add(seq)
            call, arg, admitted = "add", seq.name, []
        elif u < 0.7:
            call, arg = "admit", -1
            admitted = [q.name for q in sched.admit_ready()]
        else:
            seq = seqs[int(rng.integers(len(seqs)))]
            sched.release(seq)
            call, arg, admitted = "release", seq.name, []
        calls.append({"call": call, "arg": arg, "admitted": admitted,
                      "active": [q.name for q in sched.active_sequences()],
                      "status": [q.status.name for q in seqs]})
    return {"calls": np.array(json.dumps(calls))}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    install_librosa_stub()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    np.savez_compressed(os.path.join(HERE, "cache_window_small.npz"),
                        **cache_window_fixture((70, 1), 16, 45, 3, 2, 21))
    np.savez_compressed(os.path.join(HERE, "cache_window_large.npz"),
                        **cache_window_fixture((70, 13), 8, 9, 2, 2, 22))
    np.savez_compressed(os.path.join(HERE, "masks.npz"), **masks_fixture())
    np.savez_compressed(os.path.join(HERE, "scheduler_slots.npz"), **scheduler_fixture())
    np.savez_compressed(os.path.join(HERE, "admission.npz"), **admission_fixture())
    np.savez_compressed(os.path.join(HERE, "churn_configs4.npz"), **churn_fixture())
    np.savez_compressed(os.path.join(HERE, "encoder_small.npz"),
                        **run_encoder_fixture(None, SMALL_SCHEDULE))
    np.savez_compressed(os.path.join(HERE, "encoder_large.npz"),
                        **run_encoder_fixture(None, LARGE_SCHEDULE))
    for cfg, name in ((SMALL_FULL, "encoder_small_full.npz"), (LARGE_FULL, "encoder_large_full.npz")):
        fx = run_encoder_fixture(None, cfg)
        bf = run_encoder_fixture(None, cfg, torch.bfloat16)
        for s in cfg["keep_steps"]:
            n = fx[f"len_{s}"]
            a = np.concatenate([fx[f"out_{s}"][b, :, :k].ravel() for b, k in enumerate(n)])
            b = np.concatenate([bf[f"out_{s}"][b, :, :k].ravel() for b, k in enumerate(n)])
            fx[f"ref_bf16_err_{s}"] = np.array(np.linalg.norm(a - b) / np.linalg.norm(a))
        np.savez_compressed(os.path.join(HERE, name), **fx)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
