"""Sampled-token membership check on the GPU (the drop-in for `check_members`,
src/pck/member.py:118-197).

For every row of logits and its sampled token: the token must be in range, the row free of
NaN, fewer than k logits strictly above the token's (k = 1 for greedy rows), and, for rows
with top-p < 1, the softmax mass of the kept logits above the token (kept = at least the
k-th largest) over the kept mass must stay below p plus a slack that covers the binary32
terms and binary64 sums (`member_eps32`). One launch of `pck_member_check` (one CTA per
row) replaces the reference's torch implementation; there is no CPU path.
"""

from __future__ import annotations

import math

import torch

from pck.fp import U32, U64, gamma, next_up

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}  # PCK_LOGITS_*


def member_eps32(vocab: int) -> float:
    """Bound on |computed r - r| for binary32 terms summed in binary64
    (src/pck/member.py:84-102): E = 6 u32 + V 2^-124 + gamma_{V+2}(u64) (1 + 6 u32 + V 2^-124),
    bound 2E / (1 - E) + u64."""
    tiny = math.ldexp(vocab, -124)
    e = 6 * U32 + tiny + gamma(vocab + 2, U64) * (1 + 6 * U32 + tiny)
    return 2 * e / (1 - e) + U64


def _per_row(t, rows: int, dtype: torch.dtype, device: torch.device, name: str) -> torch.Tensor:
    v = torch.as_tensor(t, device=device).reshape(-1)
    if v.numel() != rows:
        raise RuntimeError(f"{name} must have one value per row ({rows}), got {v.numel()}")
    return v.to(dtype).contiguous()


def check_members(logits: torch.Tensor, tokens, top_k=None, top_p=None, greedy=None, tol: float = 1e-4,
                  top_k_host=None) -> dict[str, torch.Tensor]:  # fmt: skip
    """`ok` (B,) bool, `above` (B,) int64 and `mass_above` (B,) float64 for logits (B, V)
    (float32, bfloat16 or float16 on a CUDA device) and tokens (B,); optional per-row
    ``top_k`` ints (V = no top-k), ``top_p`` floats (1 = none) and ``greedy`` bools.
    ``top_k_host`` is accepted for the reference's signature; the kernel never needs it
    (nothing here synchronizes the device)."""
    import pck.cuda.ops  # noqa: F401  (registers torch.ops.pck)

    del top_k_host
    if not isinstance(logits, torch.Tensor) or not logits.is_cuda:
        raise RuntimeError("logits must be a CUDA tensor")
    if logits.dim() != 2:
        raise RuntimeError("expected logits of shape (B, V)")
    if logits.dtype not in _DTYPES:
        raise RuntimeError(f"logits must be float32, bfloat16 or float16, got {logits.dtype}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    rows, vocab = logits.shape
    dev = logits.device
    tok = _per_row(tokens, rows, torch.int64, dev, "tokens")
    tk = None if top_k is None else _per_row(top_k, rows, torch.int64, dev, "top_k")
    tp = None if top_p is None else _per_row(top_p, rows, torch.float64, dev, "top_p")
    gr = None if greedy is None else _per_row(greedy, rows, torch.bool, dev, "greedy")
    slack = next_up(tol + member_eps32(vocab))
    ok, above, mass = torch.ops.pck.member_check(logits, tok, tk, tp, gr, slack)
    return {"ok": ok, "above": above, "mass_above": mass}
