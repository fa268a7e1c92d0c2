"""Rounding helpers and error constants (oracle restatement of src/pck/fp.py).

Test infrastructure only: the product computes the same constants in `pck.fp`, and
`tests/test_fp_constants.py` checks the two against each other and against the
reference's golden values.
"""

from __future__ import annotations

import math

import numpy as np

U32 = math.ldexp(1.0, -24)  # unit roundoff, binary32, round to nearest (fp.py:10)
U64 = math.ldexp(1.0, -53)  # unit roundoff, binary64, round to nearest (fp.py:13)


def bf16(values) -> np.ndarray:
    """binary32 -> bfloat16 with round-to-nearest-even, returned widened to binary32.

    Follows src/pck/fp.py:17-28: add 0x7FFF plus the parity of bit 16 to the bit pattern
    and clear the low half; NaNs are restored afterwards (the carry could turn a NaN with
    a low payload into Inf), and finite values past the range carry into +-Inf.
    """
    out = np.array(values, dtype=np.float32, copy=True)
    is_nan = np.isnan(out)
    u = out.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    u += np.uint32(0x7FFF) + lsb
    u &= np.uint32(0xFFFF0000)
    out[is_nan] = np.nan
    return out


def gamma(k: int, u: float = U32) -> float:
    """Higham's gamma_k(u) = k u / (1 - k u) (src/pck/fp.py:31-37)."""
    if k < 0:
        raise ValueError(f"k must be non-negative, got {k}")
    ku = k * u
    if ku >= 1:
        raise ValueError(f"gamma_k needs k*u < 1, got k*u = {ku}")
    return ku / (1 - ku)


def next_up(v: float, steps: int = 1) -> float:
    """`v` moved ``steps`` binary64 values towards +inf (src/pck/fp.py:54-58)."""
    for _ in range(steps):
        v = math.nextafter(v, math.inf)
    return v


def round_up_f32(v) -> np.ndarray:
    """Non-negative binary64 values stored to binary32 rounding upward, widened back to
    binary64 (src/pck/fp.py:40-51)."""
    wide = np.asarray(v, dtype=np.float64)
    if np.any(wide < 0):
        raise ValueError("round_up_f32 expects non-negative values")
    narrow = wide.astype(np.float32)
    below = narrow.astype(np.float64) < wide
    narrow[below] = np.nextafter(narrow[below], np.float32(np.inf))
    return narrow.astype(np.float64)


def sum_up_factor(terms: int) -> float:
    """Multiplier turning a round-to-nearest binary64 sum of ``terms`` non-negative values
    into an upper bound of the exact sum: next_up(1 + 2 gamma_terms(u64))
    (src/pck/fp.py:61-66)."""
    return next_up(1.0 + 2.0 * gamma(max(terms, 1), U64))


def sum_up(s, terms: int) -> np.ndarray:
    """Upper bounds for exact sums whose binary64 nearest-rounded values are ``s``
    (src/pck/fp.py:69-73): multiply by `sum_up_factor`, then step up once."""
    wide = np.asarray(s, dtype=np.float64)
    with np.errstate(over="ignore"):
        return np.nextafter(wide * sum_up_factor(terms), np.inf)


def softmax_eps(vocab: int, zmax: float = 0.0) -> float:
    """Error bound of a binary64 softmax mass over ``vocab`` logits (src/pck/fp.py:76-99).

    E = 1.01 (V u/e + 2 zmax u + 4u) + 1.01 gamma_V(u) with u = u64, required <= 0.01;
    the mass bound is (2E + gamma_{V+2}(u)(1 + E)) / (1 - E) + 2u.
    """
    u = U64
    v = max(vocab, 1)
    big_e = 1.01 * (v * u / math.e + 2.0 * zmax * u + 4.0 * u) + 1.01 * gamma(v, u)
    if not big_e <= 0.01:
        raise ValueError(
            f"softmax over {vocab} logits with |logit / T| up to {zmax} is too "
            "large to check in FP64"
        )
    return (2.0 * big_e + gamma(v + 2, u) * (1.0 + big_e)) / (1.0 - big_e) + 2.0 * u


def ceil_div(a: int, b: int) -> int:
    """Ceiling of a / b for a >= 0, b > 0 (src/pck/fp.py:102-104)."""
    return -(-a // b)


def tree_height(n: int, threads: int, vec: int = 1) -> int:
    """Summation-tree height of the GEMV models (src/pck/fp.py:107-124).

    A thread's chain holds vec * ceil(ceil(n / vec) / threads) terms (padding included),
    i.e. that many minus one additions, and log2(threads) halving levels follow.
    """
    if n < 1:
        raise ValueError(f"n must be positive, got {n}")
    if threads < 1 or threads & (threads - 1):
        raise ValueError(f"threads must be a power of two, got {threads}")
    if vec < 1:
        raise ValueError(f"vec must be positive, got {vec}")
    chain = vec * ceil_div(ceil_div(n, vec), threads)
    return chain - 1 + (threads.bit_length() - 1)
