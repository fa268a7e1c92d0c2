"""Bit-faithful CPU models of the GEMV summation trees (oracle restatement of
src/pck/gemv.py). Test infrastructure only.

Every model takes W and x as binary32 arrays holding bfloat16 (or E4M3) values, so each
product w*x is exact in binary32 except where it underflows; the models form the products
in binary32 exactly as the kernels do, then add them in the kernel's order.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from oracle.fp import bf16, ceil_div

WARP = 32


def _products(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    m, n = W.shape
    if x.shape != (n,):
        raise ValueError(f"x has shape {x.shape}, expected ({n},)")
    return (W.astype(np.float32) * x.astype(np.float32)).astype(np.float32)


def emulate_gemv(
    W: np.ndarray,
    x: np.ndarray,
    threads: int,
    *,
    acc_bf16: bool = False,
    partial_bf16: bool = False,
    drop_tail: int = 0,
) -> np.ndarray:
    """The naive kernel's order (src/pck/gemv.py:14-57): thread t owns the contiguous
    columns [t*chunk, (t+1)*chunk), chunk = ceil(n/threads), padded with +0; the per-thread
    partials are then combined by the pairwise tree t += t + stride, stride = 1, 2, 4, ...

    The planted shortcuts (all outside the accuracy spec): ``acc_bf16`` rounds the running
    accumulator to bfloat16 after every addition, ``partial_bf16`` rounds the per-thread
    partials to bfloat16 before the tree, ``drop_tail`` zeroes the last columns.
    """
    if threads < 1 or threads & (threads - 1):
        raise ValueError(f"threads must be a power of two, got {threads}")
    P = _products(W, x)
    m, n = P.shape
    if not 0 <= drop_tail <= n:
        raise ValueError(f"drop_tail must be in [0, {n}], got {drop_tail}")
    if drop_tail:
        P[:, n - drop_tail :] = 0
    chunk = ceil_div(n, threads)
    padded = np.zeros((m, threads * chunk), dtype=np.float32)
    padded[:, :n] = P
    chains = padded.reshape(m, threads, chunk)
    acc = chains[:, :, 0].copy()
    for step in range(1, chunk):
        acc = (acc + chains[:, :, step]).astype(np.float32)
        if acc_bf16:
            acc = bf16(acc)
    if partial_bf16:
        acc = bf16(acc)
    # adjacent pairs first: (0,1), (2,3), ... then (0,2), (4,6), ...
    while acc.shape[1] > 1:
        acc = (acc[:, 0::2] + acc[:, 1::2]).astype(np.float32)
    return acc[:, 0]


def halving_sum(a: np.ndarray) -> np.ndarray:
    """Reduce the last axis (a power of two long) by a[i] += a[i + len/2], len/2 = L/2,
    L/4, ..., 1 — the order of a shuffle-down reduction (src/pck/gemv.py:60-68)."""
    while a.shape[-1] > 1:
        h = a.shape[-1] // 2
        a = (a[..., :h] + a[..., h:]).astype(np.float32)
    return a[..., 0]


def chain_columns(n: int, threads: int, vec: int) -> np.ndarray:
    """Column of every chain term of the coalesced tree, shape (threads, chain length).

    Chain t holds the vectors t, t + threads, t + 2*threads, ... of ``vec`` consecutive
    columns, in that order (src/pck/gemv.py:71-101). Columns >= n are padding (+0).
    """
    per_thread = ceil_div(ceil_div(n, vec), threads)
    v = np.arange(per_thread)[None, :, None]
    t = np.arange(threads)[:, None, None]
    k = np.arange(vec)[None, None, :]
    return ((v * threads + t) * vec + k).reshape(threads, per_thread * vec)


def emulate_gemv_coalesced(
    W: np.ndarray, x: np.ndarray, threads: int, vec: int = 8
) -> np.ndarray:
    """The coalesced kernel's order (src/pck/gemv.py:71-101): chain t adds its terms
    sequentially (the first term is taken as is), each group of 32 chains is reduced by
    halving, and the threads/32 group sums are reduced by halving again."""
    if threads < WARP or threads & (threads - 1):
        raise ValueError(f"threads must be a power of two >= {WARP}, got {threads}")
    if vec < 1:
        raise ValueError(f"vec must be positive, got {vec}")
    P = _products(W, x)
    m, n = P.shape
    cols = chain_columns(n, threads, vec)
    padded = np.zeros((m, int(cols.max()) + 1), dtype=np.float32)
    padded[:, :n] = P
    terms = padded[:, cols]  # (m, threads, chain)
    acc = terms[:, :, 0].copy()
    for step in range(1, terms.shape[2]):
        acc = (acc + terms[:, :, step]).astype(np.float32)
    group_sums = halving_sum(acc.reshape(m, threads // WARP, WARP))
    return halving_sum(group_sums)


def reference_gemv(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    """binary64 W x (src/pck/gemv.py:104-106)."""
    return W.astype(np.float64) @ x.astype(np.float64)


def abs_row_sums(W: np.ndarray, x: np.ndarray) -> np.ndarray:
    """sum_j |W_ij x_j| in binary64 (src/pck/gemv.py:109-111)."""
    return np.abs(W).astype(np.float64) @ np.abs(x).astype(np.float64)


# ---------------------------------------------------------------------------------------
# The same coalesced model in C (oracle/gemv_ref.c), for full-size shapes and the timed
# CPU baseline. Built by oracle/build.py into oracle/_build/liboracle.so.

_LIB = None


def c_library() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = Path(__file__).parent / "_build" / "liboracle.so"
        if not path.exists():
            from oracle.build import build

            build()
        lib = ctypes.CDLL(str(path))
        lib.oracle_gemv_coalesced.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
            ctypes.c_int,
        ]  # fmt: skip
        lib.oracle_gemv_coalesced.restype = ctypes.c_int
        lib.oracle_max_threads.restype = ctypes.c_int
        _LIB = lib
    return _LIB


WEIGHT_BF16, WEIGHT_E4M3 = 0, 1


def gemv_coalesced_c(
    W_bits: np.ndarray,
    X_bits: np.ndarray,
    threads: int,
    vec: int,
    weight_format: int = WEIGHT_BF16,
    cpu_threads: int | None = None,
) -> np.ndarray:
    """Y (B, m) binary32 for W (m, n) given as raw bits (uint16 bfloat16 or uint8 E4M3) and
    X (B, n) or (n,) as raw bfloat16 bits; same tree as `emulate_gemv_coalesced`."""
    lib = c_library()
    W_bits = np.ascontiguousarray(W_bits)
    X = np.ascontiguousarray(X_bits, dtype=np.uint16)
    squeeze = X.ndim == 1
    X2 = X.reshape(1, -1) if squeeze else X
    m, n = W_bits.shape
    batch = X2.shape[0]
    if X2.shape[1] != n:
        raise ValueError("X and W disagree on n")
    expected = np.uint16 if weight_format == WEIGHT_BF16 else np.uint8
    if W_bits.dtype != expected:
        raise ValueError(f"W_bits must be {np.dtype(expected).name}")
    Y = np.empty((batch, m), dtype=np.float32)
    nthreads = cpu_threads or lib.oracle_max_threads()
    rc = lib.oracle_gemv_coalesced(
        W_bits.ctypes.data, weight_format, X2.ctypes.data, Y.ctypes.data,
        m, n, batch, threads, vec, nthreads,
    )  # fmt: skip
    if rc != 0:
        raise ValueError(f"oracle_gemv_coalesced rejected its arguments (code {rc})")
    return Y[0] if squeeze else Y


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
