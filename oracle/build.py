"""TEST INFRASTRUCTURE ONLY: builds the oracle's C helpers (``oracle_c.c``)
into ``oracle/_build/liboracle.so`` with strict IEEE flags.

``__graft_entry__.build()`` calls ``build()``; the oracle also builds on first
use when the library is missing.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "oracle_c.c"
FLAGS = ["-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fexcess-precision=standard"]


def library_path() -> Path:
    return HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    out = library_path()
    if out.is_file() and not force and out.stat().st_mtime >= SOURCE.stat().st_mtime:
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    subprocess.run(["gcc", *FLAGS, str(SOURCE), "-o", str(tmp), "-lm"], check=True)
    tmp.replace(out)
    return out


if __name__ == "__main__":
    print(build(force=True))
