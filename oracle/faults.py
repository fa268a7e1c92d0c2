"""Fault models, CPU oracle (restatement of src/pck/faults.py). Test infrastructure only."""

from __future__ import annotations

import numpy as np


def flip_bit(y: np.ndarray, index: int, bit: int) -> np.ndarray:
    """Copy of binary32 ``y`` with bit ``bit`` of element ``index`` flipped
    (src/pck/faults.py:9-20): bits 0-22 mantissa, 23-30 exponent, 31 sign."""
    if y.dtype != np.float32:
        raise TypeError(f"flip_bit expects float32, got {y.dtype}")
    if not 0 <= bit < 32:
        raise ValueError(f"bit must be in [0, 32), got {bit}")
    out = y.copy()
    out.view(np.uint32)[index] ^= np.uint32(1 << bit)
    return out


def sharded_topk(logits: np.ndarray, k: int, shards: int, per_shard: int) -> np.ndarray:
    """Approximate top-k (src/pck/faults.py:23-42): the ``per_shard`` largest of each of
    ``shards`` contiguous shards, then the k largest of those; ties by index."""
    a = np.asarray(logits, dtype=np.float32)
    if not 1 <= k <= a.size or shards < 1 or per_shard < 1:
        raise ValueError("need 1 <= k <= len(logits), shards >= 1 and per_shard >= 1")
    pool = []
    for idx in np.array_split(np.arange(a.size), shards):
        if idx.size:
            order = np.lexsort((idx, -a[idx].astype(np.float64)))
            pool.append(idx[order[:per_shard]])
    cand = np.concatenate(pool)
    order = np.lexsort((cand, -a[cand].astype(np.float64)))
    return cand[order[:k]].astype(np.int64)
