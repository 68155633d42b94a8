"""Copies the reference's real-logit test set into tests/golden/ (run in a
container where the reference checkout exists; the GPU box only reads the
copies):

* qwen3_8b_8x8.npz: the reference's 64-row capture of Qwen3-8B bf16 logits
  (results/logits/qwen3-8b-8x8.npz: logits_bf16 as int16 bits, sequence,
  step, position, sampled), the rows its agreement benchmark's "8x8" cells
  use (bench/agreement.py:27-28);
* reference_outputs_8x8_{rtx4090,a10}.npz: the reference fused path's raw
  outputs on those cells on two GPUs (results/a10/rtx4090/outputs-8x8-rtx4090.npz,
  results/a10/check/outputs-8x8-a10.npz), keyed "<params>-<R>x<D>-<field>".

    python tests/golden/make_real_logits.py /path/to/reference
"""
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
FILES = {
    "results/logits/qwen3-8b-8x8.npz": "qwen3_8b_8x8.npz",
    "results/a10/rtx4090/outputs-8x8-rtx4090.npz": "reference_outputs_8x8_rtx4090.npz",
    "results/a10/check/outputs-8x8-a10.npz": "reference_outputs_8x8_a10.npz",
}


def main(reference: Path) -> None:
    for src, dst in FILES.items():
        shutil.copyfile(reference / src, HERE / dst)
        with np.load(HERE / dst) as f:
            print(dst, {k: f[k].shape for k in f.files if not k.startswith(("qwen-", "top_p-", "temperature-"))})


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference"))
