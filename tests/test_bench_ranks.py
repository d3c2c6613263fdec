"""The benchmark's multi-rank logic on CPU (gloo, world size 2).

Under torchrun every rank times its own share of streams on its own GPU with
no data-path collective; the only collectives are a barrier and one
all-reduce of the timings.  These tests run that host logic as two gloo
ranks: every rank ends with the slowest rank's time, the whole-job value is
world x per-rank units / that time, and the reference arm does its work on
rank 0 only.
"""
from __future__ import annotations

import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, times: list, out_dir: str) -> None:
    import datetime
    import json

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dist.barrier()
        ms = bench.max_over_ranks(dist, times[rank], device="cpu")
        # a second collective in the same order on every rank
        again = bench.max_over_ranks(dist, times[rank] / 2, device="cpu")
        dist.barrier()
    finally:
        dist.destroy_process_group()
    value = bench.weak_scaling_value(world, 1.12 * 64, ms)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump({"ms": ms, "again": again, "value": value}, f)


def test_every_rank_gets_the_slowest_time_and_the_whole_job_value(tmp_path):
    import json

    import torch.multiprocessing as mp
    times = [3.0, 5.5]
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, times, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    for r in res:
        assert r["ms"] == 5.5
        assert r["again"] == 2.75
        # two ranks of 64 streams x 1.12 s each in 5.5 ms
        assert r["value"] == pytest.approx(2 * 64 * 1.12 / 5.5e-3)


def test_single_process_helpers():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(None, 4.25) == 4.25
    assert bench.weak_scaling_value(1, 676724736, 1.0) == pytest.approx(676724736e3)
    assert bench.weak_scaling_value(8, 1.0, 2.0) == pytest.approx(4000.0)


def test_reference_arm_works_on_rank_zero_only():
    """Ranks other than 0 return without timing anything (no line printed)."""
    sys.path.insert(0, ROOT)
    import argparse

    import bench
    args = argparse.Namespace(workload="block", warmup=3, steps=1, gpus=2, no_encoder=True,
                              cpu_seconds=0.1, chunks_per_step=54)
    assert bench.run_reference(args, rank=1) is None


def test_reference_arm_uses_every_host_core_under_torchrun_settings():
    """torchrun sets OMP_NUM_THREADS=1 in every rank; the reference arm still
    times the oracle on all the host cores it may use, and reports them."""
    import json
    import subprocess
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--blocks", "1", "--steps", "1", "--warmup", "3", "--no-encoder"],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    cores = len(os.sched_getaffinity(0))
    assert line["impl"] == "reference" and line["cpu_baseline"]["cores"] == cores
    assert line["cpu_baseline"]["kind"] == "port" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["config"]["chunks_per_step"] == 54
