"""Rounding constants of the checked decode path (the host side of src/pck/fp.py).

These are the scalars the GPU checkers need, computed on the host and rounded outward:
unit roundoffs, Higham's gamma_k, directed steps, the summation-tree height of the GEMV
kernels, and the softmax error bound of the sampling checks.
"""

from __future__ import annotations

import math

import numpy as np

U32: float = math.ldexp(1.0, -24)
"""Unit roundoff of binary32 (round to nearest)."""

U64: float = math.ldexp(1.0, -53)
"""Unit roundoff of binary64 (round to nearest)."""


def bf16(a) -> np.ndarray:
    """binary32 values rounded to bfloat16 (nearest, ties to even), returned as binary32.
    NaN stays NaN; finite values beyond the range round to +-Inf (src/pck/fp.py:17-28)."""
    v = np.array(a, dtype=np.float32, copy=True)
    nan = np.isnan(v)
    u = v.view(np.uint32)
    u += np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    u &= np.uint32(0xFFFF0000)
    v[nan] = np.nan
    return v


def gamma(k: int, u: float = U32) -> float:
    """gamma_k(u) = k u / (1 - k u), the bound of k chained roundings (src/pck/fp.py:31-37)."""
    if k < 0:
        raise ValueError(f"k must be non-negative, got {k}")
    if k * u >= 1:
        raise ValueError(f"gamma_k needs k*u < 1, got k*u = {k * u}")
    return k * u / (1 - k * u)


def next_up(v: float, steps: int = 1) -> float:
    """``v`` moved ``steps`` binary64 values towards +inf (src/pck/fp.py:54-58)."""
    for _ in range(steps):
        v = math.nextafter(v, math.inf)
    return v


def sum_up_factor(terms: int) -> float:
    """Factor bounding an exact sum of ``terms`` non-negative values from above given its
    round-to-nearest binary64 value: next_up(1 + 2 gamma_terms(u64)) (src/pck/fp.py:61-66)."""
    return next_up(1.0 + 2.0 * gamma(max(terms, 1), U64))


def softmax_eps(vocab: int, zmax: float = 0.0) -> float:
    """Error bound of a binary64 softmax mass over ``vocab`` logits (src/pck/fp.py:76-99)."""
    u = U64
    v = max(vocab, 1)
    e = 1.01 * (v * u / math.e + 2.0 * zmax * u + 4.0 * u) + 1.01 * gamma(v, u)
    if not e <= 0.01:
        raise ValueError(
            f"softmax over {vocab} logits with |logit / T| up to {zmax} is too "
            "large to check in FP64"
        )
    return (2.0 * e + gamma(v + 2, u) * (1.0 + e)) / (1.0 - e) + 2.0 * u


def ceil_div(a: int, b: int) -> int:
    """ceil(a / b) for a >= 0 and b > 0."""
    return -(-a // b)


def tree_height(n: int, threads: int, vec: int = 1) -> int:
    """Height of the GEMV summation tree (src/pck/fp.py:107-124): a chain of
    vec * ceil(ceil(n / vec) / threads) terms, then log2(threads) halving levels."""
    if n < 1:
        raise ValueError(f"n must be positive, got {n}")
    if threads < 1 or threads & (threads - 1):
        raise ValueError(f"threads must be a power of two, got {threads}")
    if vec < 1:
        raise ValueError(f"vec must be positive, got {vec}")
    terms = vec * ceil_div(ceil_div(n, vec), threads)
    return terms - 1 + threads.bit_length() - 1
