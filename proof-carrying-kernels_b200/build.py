"""Builds libpck_b200.so, the sm_100a CUDA library behind `pck.cuda`, in the source tree.

    python proof-carrying-kernels_b200/build.py [--force]

Every translation unit under csrc/ is compiled by nvcc for sm_100a only, in parallel, and
linked into pck/_lib/libpck_b200.so (CUDA runtime linked statically). The trusted
arithmetic relies on the flags: no FMA contraction (--fmad=false), IEEE division and
square root, no flush-to-zero, warnings as errors.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
OUT_DIR = PACKAGE / "pck" / "_lib"
LIBRARY = OUT_DIR / "libpck_b200.so"
BUILD_DIR = PACKAGE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--fmad=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
    "-Werror=all-warnings",
    "-Xcompiler", "-fPIC,-Wall,-Werror",
    f"-I{INCLUDE}",
]  # fmt: skip

# Flags that would break the proven rounding model; the test suite checks they are absent.
FORBIDDEN_FLAGS = ("--use_fast_math", "-use_fast_math", "-ftz=true", "-prec-div=false",
                   "-prec-sqrt=false", "--fmad=true", "-fmad=true")  # fmt: skip


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objects = []
    jobs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(workers) as pool:
            results = list(pool.map(lambda cmd: subprocess.run(cmd, capture_output=True, text=True), jobs))
        failed = [(cmd, r) for cmd, r in zip(jobs, results, strict=True) if r.returncode != 0]
        for cmd, r in zip(jobs, results, strict=True):
            if verbose or r.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        if failed:
            raise RuntimeError(f"nvcc failed for {len(failed)} translation unit(s)")
    if force or jobs or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
            raise RuntimeError("linking libpck_b200.so failed")
        tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
