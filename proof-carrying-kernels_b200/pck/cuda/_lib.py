"""ctypes binding of libpck_b200.so (the C ABI declared in include/pck_b200.h).

The library is built in the source tree (proof-carrying-kernels_b200/build.py). There is
no fallback: if it is missing or fails to load, every GPU entry point raises.
"""

from __future__ import annotations

import ctypes
import functools
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent.parent / "_lib" / "libpck_b200.so"

PCK_OK = 0
PCK_WEIGHTS_BF16 = 0
PCK_WEIGHTS_E4M3 = 1
PCK_WEIGHTS_SETTLED = 0x100  # weights written before the preceding kernel began
PCK_CHECK_BANK_SETTLED = 0x1  # check flag: bank (c, a) written before the preceding kernel began
PCK_TC_FULL_K = 0x200  # tensor-core GEMV: one accumulation chain over the whole K per output
MAX_JOBS = 16  # PCK_MAX_JOBS
MAX_BATCH = 16
STATIC_SCRATCH_BYTES = 4 << 20  # PCK_STATIC_SCRATCH_BYTES

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_f64 = ctypes.c_double


class CheckDesc(ctypes.Structure):
    """pck_check_desc."""

    _fields_ = [
        ("c", _p), ("a", _p), ("r", _p), ("x", _p), ("y", _p),
        ("partial_cx", _p), ("partial_s", _p), ("counters", _p),
        ("passed", _p), ("rho", _p), ("tau", _p),
        ("n", _i64), ("block", _i32), ("num_blocks", _i32), ("checks", _i32),
        ("segments", _i32), ("batch", _i32), ("flags", _i32),
        ("coef", _f64), ("geps", _f64), ("tau_floor", _f64), ("c64", _p),
    ]  # fmt: skip


class GemvJob(ctypes.Structure):
    """pck_gemv_job."""

    _fields_ = [
        ("W", _p), ("X", _p), ("Y", _p), ("m", _i64), ("n", _i64),
        ("batch", _i32), ("threads", _i32), ("weight_format", _i32),
        ("w_exp_min", ctypes.c_int16), ("w_exp_max", ctypes.c_int16),
        ("check", ctypes.POINTER(CheckDesc)),
    ]  # fmt: skip


PEER_MAX_RANKS = 8
PEER_HANDLE_BYTES = 64


class PeerGather(ctypes.Structure):
    """pck_peer_gather."""

    _fields_ = [
        ("buffers", _p * PEER_MAX_RANKS), ("local", _p), ("gathered", _p),
        ("slice_bytes", _i64), ("rank", _i32), ("world", _i32),
    ]  # fmt: skip


_SIGNATURES = {
    "pck_last_error": ([], ctypes.c_char_p),
    "pck_abi_version": ([], _int),
    "pck_source_digest": ([], ctypes.c_char_p),
    "pck_device_status": ([ctypes.POINTER(ctypes.c_uint), _int], _int),
    "pck_gemv_naive": ([_p, _p, _p, _i64, _i64, _int, _p], _int),
    "pck_gemv_coalesced": ([_p, _p, _p, _i64, _i64, _int, _p], _int),
    "pck_gemv_fp8": ([_p, _p, _p, _i64, _i64, _int, _p], _int),
    "pck_gemv_batched": ([_int, _p, _p, _p, _i64, _i64, _i64, _int, _p], _int),
    "pck_blocked_check": ([ctypes.POINTER(CheckDesc), _int, _p], _int),
    "pck_gemv_checked": ([ctypes.POINTER(GemvJob), _int, _p], _int),
    "pck_gemv_checked_static": ([ctypes.POINTER(GemvJob), _int, _p], _int),
    "pck_gemv_tc": ([ctypes.POINTER(GemvJob), _int, _p], _int),
    "pck_gemv_partials": ([ctypes.POINTER(GemvJob), _int, _p], _int),
    "pck_check_verdicts": ([ctypes.POINTER(CheckDesc), _int, _p], _int),
    "pck_gemv_pipelined": ([ctypes.POINTER(GemvJob), _int, ctypes.POINTER(CheckDesc), _int, _p], _int),
    "pck_gemv_pipelined_next": ([ctypes.POINTER(GemvJob), _int, ctypes.POINTER(CheckDesc), _int,
                                 ctypes.POINTER(GemvJob), _int, _p], _int),
    "pck_sampling_check": ([_p, _p, _p, _i64, _i64, _i64, _i64, _int, _f64, _f64, _f64, _i64, _p, _p, _p, _p,
                            _p, _p], _int),
    "pck_member_check": ([_p, _int, _i64, _i64, _i64, _p, _p, _p, _p, _f64, _p, _p, _p, _p], _int),
    "pck_bank_build": ([_p, _p, _p, _p, _i64, _i64, _int, _int, _f64, _p], _int),
    "pck_sample_topk_topp": ([_p, _i64, _i64, _i64, _i64, _f64, _f64, _p, _p, _f64, _p, _p, _p], _int),
    "pck_peer_buffer_bytes": ([_i64, _int], _i64),
    "pck_peer_alloc": ([_i64, ctypes.POINTER(_p)], _int),
    "pck_peer_free": ([_p], _int),
    "pck_peer_export": ([_p, _p], _int),
    "pck_peer_import": ([_p, ctypes.POINTER(_p)], _int),
    "pck_peer_close": ([_p], _int),
    "pck_peer_all_gather": ([ctypes.POINTER(PeerGather), _p], _int),
}

EXPORTED = tuple(_SIGNATURES)


@functools.cache
def library() -> ctypes.CDLL:
    """The loaded library, with argument types set (raises if it is not built)."""
    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY} is not built; run `python proof-carrying-kernels_b200/build.py` "
            "(or __graft_entry__.build())"
        )
    lib = ctypes.CDLL(str(LIBRARY))
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


def check(rc: int, what: str = "pck") -> None:
    """Raises RuntimeError with the library's message for a non-zero status."""
    if rc != PCK_OK:
        msg = library().pck_last_error().decode(errors="replace")
        raise RuntimeError(msg or f"{what} failed with status {rc}")


def device_status(clear: bool = True) -> int:
    """The device status word (bit 0: a bounded wait in a kernel gave up). Synchronizes."""
    value = ctypes.c_uint(0)
    check(library().pck_device_status(ctypes.byref(value), int(clear)), "pck_device_status")
    return int(value.value)
