"""Builds oracle/_build/liboracle.so from oracle/gemv_ref.c (gcc, OpenMP).

Test infrastructure only. The flags keep binary32 arithmetic exact to the model: no fast
math, no contraction of a*b + c into an FMA.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
FLAGS = ["-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c11"]


def build() -> Path:
    out_dir = HERE / "_build"
    out_dir.mkdir(exist_ok=True)
    out = out_dir / "liboracle.so"
    src = HERE / "gemv_ref.c"
    if out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    tmp = out_dir / "liboracle.so.tmp"
    subprocess.run(["gcc", *FLAGS, str(src), "-o", str(tmp), "-lm"], check=True)
    tmp.replace(out)
    return out


if __name__ == "__main__":
    print(build())
