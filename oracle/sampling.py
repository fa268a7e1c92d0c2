"""Top-k / top-p set checks and reference samplers, CPU oracle (restatement of
src/pck/sampling.py). Test infrastructure only.

A selection is valid for top-k iff it is k distinct in-range indices and every selected
logit is >= every rejected logit (no NaN anywhere). For top-p it must also be minimal:
mass(S) >= p - slack and mass(S without its smallest logit) < p + slack, masses from a
binary64 softmax, slack = tol + softmax_eps rounded outward.
"""

from __future__ import annotations

import math

import numpy as np

from oracle.fp import next_up, softmax_eps


def _row(logits) -> np.ndarray:
    a = np.asarray(logits, dtype=np.float32)
    if a.ndim != 1 or a.size == 0:
        raise ValueError("logits must be a non-empty 1-D array")
    return a


def _descending_order(a: np.ndarray) -> np.ndarray:
    """Indices by decreasing logit, ties by increasing index."""
    return np.lexsort((np.arange(a.size), -a.astype(np.float64)))


def topk_reference(logits, k: int) -> np.ndarray:
    """src/pck/sampling.py:38-44."""
    a = _row(logits)
    if not 1 <= k <= a.size:
        raise ValueError(f"k must be in [1, {a.size}], got {k}")
    return _descending_order(a)[:k].astype(np.int64)


def softmax64(logits, temperature: float = 1.0) -> np.ndarray:
    """src/pck/sampling.py:47-54."""
    if not temperature > 0:
        raise ValueError(f"temperature must be positive, got {temperature}")
    z = _row(logits).astype(np.float64) / temperature
    e = np.exp(z - np.max(z))
    return e / e.sum()


def topp_reference(logits, p: float, temperature: float = 1.0) -> np.ndarray:
    """src/pck/sampling.py:57-66."""
    if not 0 < p <= 1:
        raise ValueError(f"p must be in (0, 1], got {p}")
    a = _row(logits)
    order = _descending_order(a)
    cumulative = np.cumsum(softmax64(a, temperature)[order])
    count = int(np.searchsorted(cumulative, p)) + 1
    return order[: min(count, a.size)].astype(np.int64)


def selection_mask(size: int, selected) -> np.ndarray | None:
    """src/pck/sampling.py:69-78: None unless a non-empty set of distinct in-range ints."""
    s = np.asarray(selected)
    if s.ndim != 1 or s.size == 0 or not np.issubdtype(s.dtype, np.integer):
        return None
    if s.min() < 0 or s.max() >= size or np.unique(s).size != s.size:
        return None
    mask = np.zeros(size, dtype=bool)
    mask[s] = True
    return mask


def is_prefix(a: np.ndarray, mask: np.ndarray) -> bool:
    """src/pck/sampling.py:81-87."""
    if np.isnan(a).any():
        return False
    if mask.all():
        return True
    return bool(a[mask].min() >= a[~mask].max())


def check_topk(logits, selected, k: int) -> bool:
    """src/pck/sampling.py:90-94."""
    a = _row(logits)
    mask = selection_mask(a.size, selected)
    return mask is not None and int(mask.sum()) == k and is_prefix(a, mask)


def check_topp(logits, selected, p: float, temperature: float = 1.0, tol: float = 1e-6) -> bool:
    """src/pck/sampling.py:97-122."""
    if not 0 < p <= 1:
        raise ValueError(f"p must be in (0, 1], got {p}")
    if tol < 0:
        raise ValueError(f"tol must be non-negative, got {tol}")
    a = _row(logits)
    mask = selection_mask(a.size, selected)
    if mask is None or not is_prefix(a, mask):
        return False
    probs = softmax64(a, temperature)
    mass = float(probs[mask].sum())
    sel = np.flatnonzero(mask)
    smallest = sel[np.argmin(a[sel])]
    without = mass - float(probs[smallest])
    finite = np.isfinite(a)
    zmax = 0.0 if temperature == 1.0 else float(np.abs(a[finite] / temperature).max(initial=0.0))
    slack = next_up(tol + softmax_eps(a.size, zmax))
    low, high = math.nextafter(p - slack, -math.inf), next_up(p + slack)
    return mass >= low and without < high


def check_sampled(token: int, selected) -> bool:
    """src/pck/sampling.py:125-127."""
    return bool(np.isin(token, np.asarray(selected)))
