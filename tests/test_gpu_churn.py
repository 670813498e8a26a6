"""configs[4] on the device allocator: 256 streams arriving as a Poisson
process (20 per second), lengths uniform in 2-120 s, the page pool capped at
60 % of full demand (admission waits for pages), 1144 steps of joins and
leaves mid-batch and short final chunks.  Through the drop-in Scheduler:

* the slot ids it hands out and takes back equal the reference Scheduler's
  under the same schedule (golden churn_configs4.npz, tests/golden/make_golden.py);
* the device page table, free ring and per-slot counters equal the CPU model
  (oracle/pages.py) after every 16th step and at the end, bit for bit."""
import numpy as np
import pytest
import torch

from oracle import pages
from parakeet_b200.engine import Scheduler
from parakeet_b200.ops import PagedKVPool
from replay import load, make_golden
from test_gpu_kernels import assert_pool_equals_model

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


class _Encoder:
    """What Scheduler.init_state_pool asks of an encoder: a one-layer pool
    (the allocator does not depend on the layer count or width)."""

    def make_pool(self, num_slots, device, dtype, **kw):
        return PagedKVPool(1, 128, 2, (70, 1), num_slots, dtype=dtype, device=device, **kw)


def test_configs4_churn_slots_match_reference_and_pages_match_model():
    cfg = make_golden.CHURN
    g = load("churn_configs4.npz")
    left, T, ps = 70, 2, 16
    per = pages.pages_per_stream(left, T, ps)
    assert per == cfg["pages_per_stream"]
    n_slots = int(cfg["cap"] * cfg["streams"])
    n_pages = int(cfg["cap"] * cfg["streams"] * per)
    order = np.random.default_rng(1).permutation(n_pages)
    sched = Scheduler(max_active=n_slots)
    sched.init_state_pool(_Encoder(), DEV, torch.float32, n_slots, num_pages=n_pages,
                          page_order=order)
    pool = sched.pool
    model = pages.PagePoolModel(n_pages, n_slots, left, T, ps, init_order=order)
    seen = {"steps": 0, "max_live": 0}

    def release(slot):
        sched.release_state_slot(slot)
        model.release_slot(slot)

    def on_step(step, slots, lengths, released):
        ln = [T if n is None else n for n in lengths]
        sl = torch.tensor(slots, dtype=torch.int32, device=DEV)
        lt = torch.tensor(ln, dtype=torch.int32, device=DEV)
        assert model.begin_step(slots)
        pool.begin_step(sl, lt)
        model.end_step(slots, ln)
        pool.end_step(sl, lt)
        seen["steps"] = step + 1
        seen["max_live"] = max(seen["max_live"], len(slots))
        if step % 16 == 0:
            assert_pool_equals_model(pool, model)

    ops = make_golden.churn_replay(sched.acquire_state_slot, release, on_step=on_step)
    assert np.array_equal(np.array(ops, np.int64), g["ops"])
    assert seen["steps"] == int(g["steps"]) and seen["max_live"] == int(g["max_live"]) == n_slots
    assert pool.read_error() == 0
    assert_pool_equals_model(pool, model)
    assert len(model.free) == n_pages                     # every page came back
