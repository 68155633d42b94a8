"""The multi-rank host logic of bench.py on CPU (gloo, world size 2): every
rank gets the maximum of the ranks' timings, and under torchrun the reference
arm runs on rank 0 alone while the other ranks exit 0 without output.

The row-sharded GPU path has no collective on its data path (every rank runs
its own requests); these tests cover the reduction and launch logic around it.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _max_worker(rank, world, port, values, results):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        results[rank] = bench.max_over_ranks(values[rank])
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_with_two_gloo_ranks():
    import torch.multiprocessing as mp

    values = [[103.0, 7.5, 1.0], [99.0, 9.25, 2.0]]
    with mp.Manager() as manager:
        # A free port can be taken by another process before rank 0 binds it:
        # such an attempt fails at rendezvous and is retried on a new port.
        for attempt in range(3):
            results = manager.dict()
            try:
                mp.spawn(_max_worker, args=(2, _free_port(), values, results), nprocs=2, join=True)
                break
            except mp.ProcessRaisedException as e:
                if attempt == 2 or "address already in use" not in str(e).lower():
                    raise
        got = dict(results)
    assert got[0] == got[1] == [103.0, 9.25, 2.0]


def test_max_over_ranks_without_a_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks([1, 2.5]) == [1.0, 2.5]


def _bench(args, env_extra, timeout=600):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, *args], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_on_a_non_zero_rank_exits_quietly():
    done = _bench(["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                  {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert done.returncode == 0, done.stderr
    assert done.stdout.strip() == ""


@pytest.mark.slow
def test_reference_arm_under_torchrun_prints_one_line():
    done = _bench(["-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
                   "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference", "--gpus", "2",
                   "--steps", "1", "--warmup", "3", "--cpu-sample", "2"], {"OMP_NUM_THREADS": "1"})
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [l for l in done.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"


def test_sampler_grid_is_the_reference_grid():
    """bench.py --sampler-shapes runs the grid of the reference's
    bench/sampler.py:36-41: three settings by eight (requests, drafts) shapes."""
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.SAMPLER_SETTINGS == {
        "qwen": dict(temperature=0.6, top_k=20, top_p=0.95, min_p=0.0),
        "temperature": dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0),
        "top_p": dict(temperature=0.7, top_k=0, top_p=0.9, min_p=0.0),
    }
    assert bench.SAMPLER_SHAPES == [(1, 0), (8, 0), (32, 0), (128, 0), (1, 4), (8, 4), (32, 4), (64, 4)]
    done = _bench(["bench.py", "--sampler-shapes", "nonsense"], {})
    assert done.returncode != 0 and "invalid choice" in done.stderr
