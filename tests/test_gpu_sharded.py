"""Vocabulary-sharded calls on the GPU: the same outputs as the unsharded
call, on every shard, for 2 to 8 shards (shard widths that do and do not
fall on mask-word boundaries), sampling and verification, one-hot and full
proposals, masks, fp32 and bf16, and calls repeated on the same plans.

On one GPU the N shards are N plans in one process (each call's steps issued
shard by shard, so no kernel waits on another); with two or more GPUs a
torchrun job runs one shard per GPU."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from tests import cases as C
from tests import sharded_case
from tests.gpu_helpers import device_inputs, run_abi

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def _same(got, expected, context):
    names = ["tokens", "accepted_len", "status", "path_used"]
    for g, e, name in zip(got, expected, names):
        np.testing.assert_array_equal(g, e, err_msg=f"{context}: {name}")


CASES = [
    ("C2a", dict(requests=range(16))),
    ("C3a", dict(requests=range(8))),
    ("C3b_ratio_full", dict(requests=range(4))),
    ("C3b_coupled_onehot", dict(requests=range(6))),
    ("C4", dict(requests=range(19))),
]


@pytest.mark.parametrize("shards", [2, 3, 8])
@pytest.mark.parametrize("name,kw", CASES, ids=[c[0] for c in CASES])
def test_sharded_equals_unsharded(name, kw, shards):
    case = C.workload_case(name, **kw)
    expected = run_abi(device_inputs(case), mode=case["mode"])
    for rank, got in enumerate(sharded_case.emulated(case, shards)):
        _same(got, expected, f"{name} shards={shards} rank={rank}")


def test_sharded_bf16_and_repeated_calls():
    case = C.workload_case("C2a", requests=range(12))
    expected = run_abi(device_inputs(case, dtype="bfloat16"), mode=case["mode"])
    for rank, got in enumerate(sharded_case.emulated(case, 4, dtype="bfloat16", calls=3)):
        _same(got, expected, f"bf16 rank={rank}")


def test_sharded_small_cases_match_their_goldens():
    from tests import golden_io
    for case, expected in golden_io.small()[::5]:
        if case["logits"].shape[1] < 64 or case["cu_rows"].size < 2:
            continue
        for rank, got in enumerate(sharded_case.emulated(case, 2)):
            np.testing.assert_array_equal(got[2], expected[2], err_msg=f"{case['name']} rank={rank}: status")
            np.testing.assert_array_equal(got[0][:, :expected[0].shape[1]], expected[0],
                                          err_msg=f"{case['name']} rank={rank}: tokens")


def test_one_shard_per_gpu_under_torchrun():
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    n = min(n, 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    done = subprocess.run(
        ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
         f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(port),
         str(ROOT / "tests" / "sharded_worker.py")], cwd=ROOT, env=env, capture_output=True, text=True)
    assert done.returncode == 0, done.stdout[-3000:] + done.stderr[-3000:]
    assert done.stdout.count("sharded ok") == n
