"""The N>1 host path of bench.py on CPU: two gloo ranks on 127.0.0.1.

bench.py runs one replica per GPU (weak scaling, no collective on the data
path); across ranks it only takes the max of the timings and reports the
whole-job throughput on rank 0.  These tests run that host logic with the
gloo backend, and the reference arm's rank handling under a 2-rank launch.
"""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)
import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        # rank r "measured" (ms, e2e_ms, attn_ms, eager_ms)
        mine = [1.0 + rank, 5.0 - rank, 0.5 * (rank + 1), 2.0]
        got = bench.max_over_ranks(mine, torch.device("cpu"))
        dist.barrier()
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(got, f)
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo_two_ranks(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    assert res[0] == res[1] == [2.0, 5.0, 1.0, 2.0]


def test_max_over_ranks_single_process_is_identity():
    assert bench.max_over_ranks([1.5, 2.5], torch.device("cpu")) == [1.5, 2.5]


def test_job_throughput_counts_every_rank():
    # 2 ranks x 1e9 bytes per step in 1 ms (the slowest rank) = 2e12 B/s
    assert bench.job_throughput(1e9, 2, 1.0) == pytest.approx(2000.0)


def test_reference_arm_only_rank0_reports():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"],
                       env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0
    assert r.stdout.strip() == ""


def _serve_rank_main(rank, world, port, out_dir):
    """Two engines behind the router: every rank places the same 1001 streams,
    serves its share (a fake trial whose latencies depend on the rank) and
    reduces the result with the other rank."""
    import numpy as np
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        from parakeet_b200.engine import StreamRouter
        router = StreamRouter(world)
        where = [router.place(s) for s in range(1001)]
        served = []

        def local(n):
            served.append(n)
            lat = np.full(n, 0.010 * (rank + 1))           # rank 1 is slower
            return lat, {"backlog_chunks_at_end": rank, "streams_joined": 3}

        ok, rec = bench.job_trial(1001, world, rank, 10_000, torch.device("cpu"), 160.0, local)
        with open(os.path.join(out_dir, f"serve{rank}.json"), "w") as f:
            json.dump({"where": where, "served": served, "ok": ok, "rec": rec}, f)
    finally:
        dist.destroy_process_group()


def test_job_serving_trial_gloo_two_ranks(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_serve_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    res = [json.load(open(tmp_path / f"serve{r}.json")) for r in range(world)]
    assert res[0]["where"] == res[1]["where"]            # same placement on every rank
    assert res[0]["served"] == [501] and res[1]["served"] == [500]
    for r in res:                                         # both ranks see the job's result
        assert r["ok"] is True
        assert r["rec"]["p99_ms"] == pytest.approx(20.0)   # the slower rank's p99
        assert r["rec"]["chunks"] == 1001 and r["rec"]["streams_served"] == 1001
        assert r["rec"]["backlog_chunks_at_end"] == 1 and r["rec"]["streams_joined"] == 6
    assert res[0]["rec"] == res[1]["rec"]


def test_router_least_loaded_with_capacity_and_release():
    from parakeet_b200.engine import StreamRouter
    r = StreamRouter(3, capacity=2)
    assert [r.place(i) for i in range(6)] == [0, 1, 2, 0, 1, 2]
    assert r.place(6) is None                              # every engine full
    assert r.release(4) == 1 and r.place(7) == 1           # the freed engine takes the next
    r.release(0)
    r.release(3)
    assert r.load == [0, 2, 2] and r.place(8) == 0 and r.streams_of(1) == [1, 7]
    with pytest.raises(ValueError):
        r.place(8)
