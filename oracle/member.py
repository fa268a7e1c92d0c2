"""Sampled-token membership check, CPU oracle (restatement of src/pck/member.py).
Test infrastructure only.

For a row of logits l, sampled token t and the request's top-k / top-p / greedy setting:
  above = #{j : l_j > l_t};
  top-k / greedy: accept iff above < k (k = 1 when greedy);
  top-p: kept = {j : l_j >= k-th largest} (all when there is no top-k); r = (mass of kept
  tokens with l_j > l_t) / (mass of kept tokens); accept iff r < p + slack, slack =
  tol + eps rounded outward.
NaN anywhere in the row, or a token id outside [0, V), rejects.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from oracle.fp import U32, U64, gamma, next_up, softmax_eps


def member_eps(vocab: int) -> float:
    """Error of the binary64 reference fraction (src/pck/member.py:37-41)."""
    return softmax_eps(vocab)


def member_eps32(vocab: int) -> float:
    """Error of the fraction computed from binary32 terms summed in binary64
    (src/pck/member.py:84-102): E = 6 u32 + V 2^-124 + gamma_{V+2}(u64)(1 + 6 u32 + V 2^-124),
    bound 2E/(1 - E) + u64."""
    tiny = math.ldexp(vocab, -124)
    e = 6 * U32 + tiny + gamma(vocab + 2, U64) * (1 + 6 * U32 + tiny)
    return 2 * e / (1 - e) + U64


@dataclass(frozen=True)
class MemberVerdict:
    ok: bool
    above: int
    mass_above: float


def check_member(logits, token: int, top_k: int | None = None, top_p: float | None = None,
                 *, greedy: bool = False, tol: float = 1e-4) -> MemberVerdict:  # fmt: skip
    """One row, binary64 throughout (src/pck/member.py:53-81)."""
    lv = np.asarray(logits, dtype=np.float64)
    if np.isnan(lv).any() or not 0 <= token < lv.size:
        return MemberVerdict(False, -1, math.nan)
    lt = lv[token]
    above = int(np.count_nonzero(lv > lt))
    k = 1 if greedy else top_k
    if k is not None and above >= k:
        return MemberVerdict(False, above, math.nan)
    if greedy or top_p is None or top_p >= 1.0:
        return MemberVerdict(True, above, 0.0)
    if top_k is not None and top_k < lv.size:
        kth = np.sort(lv)[lv.size - top_k]
        kept = lv >= kth
    else:
        kept = np.ones(lv.shape, dtype=bool)
    top = lv[kept].max()
    e = np.where(kept, np.exp(lv - top), 0.0)
    r = float(e[lv > lt].sum() / e.sum())
    slack = next_up(tol + member_eps(lv.size))
    return MemberVerdict(bool(r < next_up(top_p + slack)), above, r)


def split_terms(x: np.ndarray, m: np.ndarray) -> np.ndarray:
    """binary32 e^(x - m) from the exact TwoSum split x - m = hi + lo
    (src/pck/member.py:105-115): expf(hi) + expf(hi)*lo, 0 where hi < -128 or NaN."""
    x = x.astype(np.float32)
    nm = (-np.asarray(m, dtype=np.float32)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        hi = (x + nm).astype(np.float32)
        bv = (hi - x).astype(np.float32)
        lo = ((x - (hi - bv)) + (nm - bv)).astype(np.float32)
        eh = np.exp(hi).astype(np.float32)
        t = (eh + (eh * lo).astype(np.float32)).astype(np.float32)
    return np.where(hi >= -128.0, t, np.float32(0.0))


def check_members(logits: np.ndarray, tokens, top_k=None, top_p=None, greedy=None,
                  tol: float = 1e-4) -> dict:  # fmt: skip
    """The batched check's outputs (src/pck/member.py:118-197), evaluated row by row in
    NumPy from its definition: `above` counts against the token id clamped into range
    (an out-of-range id still rejects), the top-p fraction uses `split_terms` summed in
    binary64, and `mass_above` is that fraction on rows with p < 1 (0 elsewhere)."""
    lv = np.asarray(logits, dtype=np.float32)
    rows, vocab = lv.shape
    tokens = np.asarray(tokens).astype(np.int64).reshape(rows)
    ok = np.zeros(rows, dtype=bool)
    above = np.zeros(rows, dtype=np.int64)
    mass = np.zeros(rows, dtype=np.float64)
    slack = next_up(tol + member_eps32(vocab))
    for i in range(rows):
        row = lv[i]
        t = int(tokens[i])
        in_range = 0 <= t < vocab
        lt = row[min(max(t, 0), vocab - 1)]
        gt = row > lt
        above[i] = int(gt.sum())
        finite = not np.isnan(row).any()
        k = vocab if top_k is None else int(min(max(int(top_k[i]), 1), vocab))
        is_greedy = bool(greedy[i]) if greedy is not None else False
        ok_k = 1 if is_greedy else k
        good = finite and in_range and above[i] < ok_k
        if top_p is not None:
            p = float(top_p[i])
            if k < vocab:
                kth = np.sort(row)[vocab - k]
                kept = row >= kth
            else:
                kept = np.ones(vocab, dtype=bool)
            x = np.where(kept, row, np.float32(-np.inf)).astype(np.float32)
            top = np.max(x)  # NaN rows give NaN, as torch's max does
            e = split_terms(x, top)
            z = math.fsum(e.astype(np.float64)) if finite else math.nan
            a = math.fsum(e[gt].astype(np.float64)) if finite else math.nan
            r = a / z if z else math.nan
            mass[i] = r if p < 1.0 else 0.0
            high = math.nextafter(p + slack, math.inf)
            good = good and (p >= 1.0 or is_greedy or r < high)
        ok[i] = good
    return {"ok": ok, "above": above, "mass_above": mass}
