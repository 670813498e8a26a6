"""Pins the CPU oracle against golden vectors produced by the reference."""
import numpy as np
import pytest

from oracle import pages, streaming
from parakeet_b200.weights import random_encoder_layers
from replay import LARGE, SMALL, SMALL_FULL, load, rel_l2, schedule, valid_rows


@pytest.mark.parametrize("name,att", [("cache_window_small.npz", (70, 1)),
                                      ("cache_window_large.npz", (70, 13))])
def test_dense_cache_matches_reference_bitexact(name, att):
    g = load(name)
    steps, layers, B, T, D = g["keys"].shape
    c = streaming.DenseModelCache(layers, att, D, 9, slots=B, dtype=np.float32)
    for s in range(steps):
        for l in range(layers):
            k, v = c.update_attn_cache(l, g["keys"][s, l], g["values"][s, l])
            assert np.array_equal(k, g["win_k"][s, l])
            assert np.array_equal(v, g["win_v"][s, l])


@pytest.mark.parametrize("name,att", [("cache_window_small.npz", (70, 1)),
                                      ("cache_window_large.npz", (70, 13))])
@pytest.mark.parametrize("page_size", [16, 8])
def test_page_model_window_equals_reference_window(name, att, page_size):
    """Pages + ring page table reproduce the reference's dense window exactly,
    with pages handed out in a scrambled order."""
    g = load(name)
    steps, layers, B, T, D = g["keys"].shape
    left = att[0]
    n = pages.pages_per_stream(left, T, page_size) * B
    order = np.random.default_rng(1).permutation(n)
    pool = pages.PagePoolModel(n, B, left, T, page_size, init_order=order)
    kv = pages.PagedKVModel(pool, layers, D, np.float32)
    slots = list(range(B))
    for s in range(steps):
        assert pool.begin_step(slots)
        for l in range(layers):
            kv.append(l, slots, g["keys"][s, l], g["values"][s, l])
            k, v = kv.gather(l, slots)
            assert np.array_equal(k, g["win_k"][s, l])
            assert np.array_equal(v, g["win_v"][s, l])
        pool.end_step(slots, [T] * B)
        held = (pool.next - pool.first)
        assert held.max() <= pages.pages_per_stream(left, T, page_size)
    assert len(pool.free) + int((pool.next - pool.first).sum()) == n


@pytest.mark.parametrize("tag", ["small", "large"])
def test_streaming_masks_match_reference(tag):
    g = load("masks.npz")
    att = (70, 1) if tag == "small" else (70, 13)
    pad, m = streaming.streaming_masks(att[1] + 1, g[f"{tag}_cache_len"],
                                       g[f"{tag}_processed"], g[f"{tag}_lengths"], att)
    assert np.array_equal(pad, g[f"{tag}_pad"])
    assert np.array_equal(m, g[f"{tag}_att"])


def test_slot_scheduler_sequence_matches_reference():
    ops = load("scheduler_slots.npz")["ops"]
    m = streaming.SlotSchedulerModel(1, (70, 1), 4, 9, 8)
    for kind, slot in ops:
        if kind == 0:
            got = m.acquire_state_slot()
            assert (-1 if got is None else got) == slot
        else:
            m.release_state_slot(int(slot))


def run_oracle_schedule(cfg):
    """The reference's runner loop (pack -> encoder -> unpack) on the oracle."""
    left, right = cfg["att"]
    sd = random_encoder_layers(cfg["seed"], cfg["layers"], cfg["dim"], cfg["heads"])
    lw = streaming.layer_weights_from_state_dict(sd, cfg["layers"])
    pe = streaming.rel_pos_table(cfg["dim"], 5000)
    sched = streaming.SlotSchedulerModel(cfg["layers"], cfg["att"], cfg["dim"], 9, cfg["pool"])
    slot_of, outs = {}, {}
    for s, rel, acq, names, x, length in schedule(cfg):
        for n in rel:
            sched.release_state_slot(slot_of[n])
        for n in acq:
            slot_of[n] = sched.acquire_state_slot()
        st, idx = sched.pack_states([slot_of[n] for n in names])
        y = streaming.encoder_step(x, st, length, lw, pe, cfg["att"], cfg["heads"])
        sched.unpack_states(st, idx)
        outs[s] = (y, length, idx)
    return outs, sched


@pytest.mark.parametrize("cfg,name", [(SMALL, "encoder_small.npz"), (LARGE, "encoder_large.npz"),
                                      (SMALL_FULL, "encoder_small_full.npz")])
def test_oracle_encoder_matches_reference_fp32(cfg, name):
    g = load(name)
    outs, sched = run_oracle_schedule(cfg)
    for s in g["keep_steps"]:
        y, length, idx = outs[int(s)]
        assert np.array_equal(idx, g[f"slots_{s}"])
        assert np.array_equal(length, g[f"len_{s}"])
        err = rel_l2(valid_rows(y, length), valid_rows(g[f"out_{s}"], length))
        assert err <= 1e-5, (s, err)
    assert np.array_equal(sched.pool.processed_frames, g["final_processed"])
    assert np.array_equal(sched.pool.cache_lengths, g["final_cache_len"])
    assert rel_l2(sched.pool.cache.conv[:, 0], g["final_conv_l0"]) <= 1e-5
