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
