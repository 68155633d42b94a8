"""One rank of the multi-GPU sharded test (run by torchrun from
tests/test_gpu_sharded.py): each rank holds one vocabulary shard, runs the
sharded call in both modes (per-phase exchange and column pulling), and
checks its outputs against the unsharded call on its own GPU and, for the
sampling case, against the CPU oracle."""
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
from tests import cases as C  # noqa: E402
from tests import sharded_case  # noqa: E402
from tests.gpu_helpers import device_inputs, run_abi  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        for name, kw in [("C2a", dict(requests=range(16))), ("C3a", dict(requests=range(8))),
                         ("C3b_ratio_full", dict(requests=range(4))), ("C4", dict(requests=range(19))),
                         ("C2b", dict(requests=range(3))), ("C3b_coupled_onehot", dict(requests=range(4)))]:
            case = C.workload_case(name, **kw)
            expected = run_abi(device_inputs(case), mode=case["mode"])
            for phases in (True, False):
                got = sharded_case.distributed(case, phases=phases, calls=2)
                for g, e in zip(got, expected):
                    np.testing.assert_array_equal(g, e, err_msg=f"{name} phases={phases} rank {dist.get_rank()}")
            if name == "C2a":
                want = oracle.verify_reference(**C.oracle_inputs(case, oracle))
                np.testing.assert_array_equal(got[2], want.status)
                np.testing.assert_array_equal(got[0][:, :1], want.tokens[:, :1])
        print("sharded ok", dist.get_rank(), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
