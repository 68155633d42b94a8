"""Builds the native libraries in-tree (no JIT cache):

* ``libexactsample_b200.so``: the CUDA kernels and the C ABI of
  ``include/exactsample_b200.h`` (nvcc, sm_100a only, --fmad=false, static
  CUDA runtime);
* ``exactsample_cuda.so``: the torch op ``exactsample::verify_out``, a thin
  shim over the C ABI (g++ against the installed torch).

    python -m exactsample_b200.build [--force]

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the
image's toolchain is present.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = PACKAGE / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [*ARCH, "-O3", "-std=c++17", "--fmad=false", "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}"]
CUDA_SOURCES = ["es_abi.cu", "es_rows_f32.cu", "es_rows_f64.cu", "es_rows_f16.cu", "es_rows_bf16.cu",
                "es_rows_full_f32.cu", "es_rows_full_f64.cu", "es_rows_full_f16.cu", "es_rows_full_bf16.cu"]
HEADERS = sorted(CSRC.glob("*.cuh")) + [INCLUDE / "exactsample_b200.h"]

CORE_LIB = PACKAGE / "libexactsample_b200.so"
TORCH_LIB = PACKAGE / "exactsample_cuda.so"
# The checked build (-DES_CHECKS: device bounds checks that count failures in
# the workspace instead of trapping), for the GPU tests' checked run.
CHECKED_LIB = PACKAGE / "libexactsample_b200_checked.so"
CHECKED_BUILD = PACKAGE / "_build_checked"


def _stale(target: Path, deps) -> bool:
    if not target.is_file():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd):
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(map(str, cmd))}\n{result.stdout}\n{result.stderr}")
    return result.stdout + result.stderr


def build_core(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    objects, jobs = [], []
    for name in CUDA_SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *HEADERS]):
            jobs.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as pool:
            for out in pool.map(_run, jobs):
                if verbose and out.strip():
                    print(out)
    if force or jobs or _stale(CORE_LIB, objects):
        tmp = CORE_LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)])
        tmp.replace(CORE_LIB)
    return CORE_LIB


def build_checked(force: bool = False) -> Path:
    """libexactsample_b200_checked.so: the C ABI library built with -DES_CHECKS."""
    CHECKED_BUILD.mkdir(exist_ok=True)
    objects, jobs = [], []
    for name in CUDA_SOURCES:
        src = CSRC / name
        obj = CHECKED_BUILD / (name + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *HEADERS]):
            jobs.append([NVCC, *NVCC_FLAGS, "-DES_CHECKS", "-c", str(src), "-o", str(obj)])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as pool:
            list(pool.map(_run, jobs))
    if force or jobs or _stale(CHECKED_LIB, objects):
        tmp = CHECKED_LIB.with_suffix(".so.tmp")
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)])
        tmp.replace(CHECKED_LIB)
    return CHECKED_LIB


def build_torch_op(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "es_torch.cpp"
    if not force and not _stale(TORCH_LIB, [src, CORE_LIB, INCLUDE / "exactsample_b200.h"]):
        return TORCH_LIB
    includes = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")] + [f"-I{CUDA_HOME / 'include'}",
                                                                                    f"-I{INCLUDE}"]
    libdirs = [f"-L{p}" for p in cpp_extension.library_paths(device_type="cuda")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=exactsample_cuda", *includes, str(src), "-o", str(tmp), *libdirs,
           f"-L{PACKAGE}", "-lexactsample_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in cpp_extension.library_paths(device_type="cuda")]]
    _run(cmd)
    tmp.replace(TORCH_LIB)
    return TORCH_LIB


def build(force: bool = False, verbose: bool = False):
    core = build_core(force, verbose)
    op = build_torch_op(force)
    checked = build_checked(force)
    return core, op, checked


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    for path in build(args.force, args.verbose):
        print(path)


if __name__ == "__main__":
    sys.exit(main())
