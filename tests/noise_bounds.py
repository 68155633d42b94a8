"""Builds tests/noise_bounds.cu (the exhaustive 2^32-word check of the FP32
noise bounds) with the library's flags, into tests/_build/noise_bounds."""
from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "noise_bounds.cu"
BINARY = HERE / "_build" / "noise_bounds"


def build(force: bool = False) -> Path:
    from exactsample_b200.build import ARCH, INCLUDE, NVCC
    deps = [SOURCE, HERE.parent / "exactsample_b200" / "csrc" / "es_device.cuh"]
    if BINARY.is_file() and not force and all(BINARY.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return BINARY
    BINARY.parent.mkdir(exist_ok=True)
    subprocess.run([NVCC, *ARCH, "-O3", "-std=c++17", "--fmad=false", f"-I{INCLUDE}", str(SOURCE), "-o",
                    str(BINARY)], check=True)
    return BINARY


if __name__ == "__main__":
    print(build(force=True))
