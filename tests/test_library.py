"""The C-ABI library: it loads, exports every entry point include/pck_b200.h declares, and
rejects bad arguments before touching a GPU. CPU only (no kernel is launched)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "pck_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pck_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from pck.cuda import _lib

    return _lib.library()


def test_header_declares_the_entry_points() -> None:
    names = declared_functions()
    assert {"pck_gemv_coalesced", "pck_gemv_fp8", "pck_blocked_check", "pck_gemv_checked"} <= set(names)


def test_library_exports_every_declared_symbol(lib) -> None:
    from pck.cuda import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIBRARY)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r" T (pck_[a-z0-9_]+)$", out.stdout, flags=re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for name in declared_functions():
        assert hasattr(lib, name)
    # the Python binding covers every declared function
    assert set(declared_functions()) == set(_lib.EXPORTED)


def test_abi_version(lib) -> None:
    assert lib.pck_abi_version() == 6


def _err(lib) -> str:
    return lib.pck_last_error().decode()


@pytest.mark.parametrize("threads", [0, 16, 48, 2048])
def test_gemv_rejects_thread_counts(lib, threads: int) -> None:
    rc = lib.pck_gemv_coalesced(1, 1, 1, 4, 8, threads, None)
    assert rc == 1 and "power of two" in _err(lib)


def test_gemv_empty_output_launches_nothing(lib) -> None:
    assert lib.pck_gemv_coalesced(None, None, None, 0, 8, 256, None) == 0
    assert lib.pck_gemv_naive(None, None, None, 0, 8, 1, None) == 0


def test_gemv_rejects_null_pointers_and_bad_batch(lib) -> None:
    assert lib.pck_gemv_coalesced(None, None, None, 4, 8, 256, None) == 1
    assert lib.pck_gemv_batched(0, 1, 1, 1, 4, 8, 17, 256, None) == 1 and "batch" in _err(lib)
    assert lib.pck_gemv_batched(7, 1, 1, 1, 4, 8, 1, 256, None) == 1 and "format" in _err(lib)


def test_blocked_check_rejects_bad_batches(lib) -> None:
    from pck.cuda import _lib

    descs = (_lib.CheckDesc * 17)()
    assert lib.pck_blocked_check(descs, 0, None) == 1 and "batch size" in _err(lib)
    assert lib.pck_blocked_check(descs, 17, None) == 1 and "batch size" in _err(lib)
    assert lib.pck_blocked_check(descs, 1, None) == 1 and "NULL" in _err(lib)
    d = descs[0]
    for f in ("c", "a", "r", "x", "y", "partial_cx", "partial_s", "counters", "passed", "rho", "tau"):
        setattr(d, f, 16)
    d.n, d.block, d.num_blocks, d.checks, d.segments, d.batch = 64, 8, 2, 1, 65, 1
    d.coef, d.geps, d.tau_floor = 1e-6, 1e-12, 1e-40
    assert lib.pck_blocked_check(descs, 1, None) == 1 and "segments" in _err(lib)
    d.segments, d.geps = 1, 0.0
    assert lib.pck_blocked_check(descs, 1, None) == 1 and "positive" in _err(lib)
    d.geps, d.flags = 1e-12, 0x2
    assert lib.pck_blocked_check(descs, 1, None) == 1 and "flags" in _err(lib)


def test_check_flag_constants_match_the_header() -> None:
    """The ctypes binding's flag values and the CheckDesc field are the header's."""
    from pck.cuda import _lib

    text = HEADER.read_text()
    for name in ("PCK_CHECK_BANK_SETTLED", "PCK_WEIGHTS_SETTLED", "PCK_TC_FULL_K"):
        m = re.search(rf"#define {name} (0x[0-9a-fA-F]+|\d+)", text)
        assert m and int(m.group(1), 0) == getattr(_lib, name), name
    assert "int32_t flags;" in text and "flags" in dict(_lib.CheckDesc._fields_)


def test_fused_check_must_cover_its_job(lib) -> None:
    from pck.cuda import _lib

    desc = _lib.CheckDesc()
    for f in ("c", "a", "r", "x", "y", "partial_cx", "partial_s", "counters", "passed", "rho", "tau"):
        setattr(desc, f, 16)
    desc.n, desc.block, desc.num_blocks, desc.checks, desc.segments, desc.batch = 64, 8, 2, 1, 1, 1
    desc.coef, desc.geps, desc.tau_floor = 1e-6, 1e-12, 1e-40
    jobs = (_lib.GemvJob * 1)()
    jobs[0].W, jobs[0].X, jobs[0].Y, jobs[0].m, jobs[0].n = 16, 32, 16, 16, 64
    jobs[0].batch, jobs[0].threads, jobs[0].weight_format = 1, 256, 0
    jobs[0].check = ctypes.pointer(desc)
    assert lib.pck_gemv_checked(jobs, 1, None) == 1 and "cover" in _err(lib)


def test_pipelined_rejects_prior_checks_sharing_its_outputs(lib) -> None:
    from pck.cuda import _lib

    prior = (_lib.CheckDesc * 1)()
    d = prior[0]
    for f in ("c", "a", "r", "x", "y", "partial_cx", "partial_s", "counters", "passed", "rho", "tau"):
        setattr(d, f, 4096)
    d.n, d.block, d.num_blocks, d.checks, d.segments, d.batch = 64, 8, 2, 1, 1, 1
    d.coef, d.geps, d.tau_floor = 1e-6, 1e-12, 1e-40
    jobs = (_lib.GemvJob * 1)()
    jobs[0].W, jobs[0].X, jobs[0].Y, jobs[0].m, jobs[0].n = 16, 32, 4096 + 32, 16, 64
    jobs[0].batch, jobs[0].threads, jobs[0].weight_format = 1, 256, 0
    assert lib.pck_gemv_pipelined(jobs, 1, prior, 1, None) == 1 and "shares memory" in _err(lib)
    assert lib.pck_gemv_pipelined(jobs, 1, prior, 17, None) == 1 and "prior" in _err(lib)
    assert lib.pck_gemv_pipelined(jobs, 1, None, 1, None) == 1 and "prior" in _err(lib)


def test_bank_build_rejects_bad_blocks(lib) -> None:
    assert lib.pck_bank_build(1, 1, 1, 1, 100, 8, 7, 1, 1.0, None) == 1 and "divide" in _err(lib)
    assert lib.pck_bank_build(1, 1, 1, 1, 64, 8, 8, 0, 1.0, None) == 1 and "checks" in _err(lib)


def test_build_flags_keep_the_rounding_model() -> None:
    """No fast math, no FMA contraction, no flush-to-zero (the flag audit of the reference's
    src/pck/cuda/ptx_audit.py:59-67)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("pck_build", ROOT / "proof-carrying-kernels_b200" / "build.py")
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    flags = build.NVCC_FLAGS
    assert "--fmad=false" in flags and "-ftz=false" in flags and "-prec-div=true" in flags
    assert not any(f in flags for f in build.FORBIDDEN_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags


def test_pipelined_next_rejects_a_bad_next_count(lib) -> None:
    """pck_gemv_pipelined_next validates its `next` jobs before any device work."""
    import ctypes

    from pck.cuda import _lib

    job = (_lib.GemvJob * 1)()
    job[0].W = job[0].X = job[0].Y = 16
    job[0].m, job[0].n, job[0].batch, job[0].threads = 128, 64, 1, 256
    job[0].check = ctypes.POINTER(_lib.CheckDesc)()
    rc = lib.pck_gemv_pipelined_next(job, 1, None, 0, job, -1, None)
    assert rc == 1 and b"next jobs" in lib.pck_last_error()
