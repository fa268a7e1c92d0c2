"""GEMV entry points (the GPU side of src/pck/cuda/gemv.py).

All of them run the sm_100a kernels of libpck_b200.so on the caller's current stream and
return binary32 outputs bit-identical to the reference's CPU models of its kernels.
"""

from __future__ import annotations

import torch

from pck.cuda._ext import extension

FP8_MAX = 448.0
"""Largest finite E4M3 value."""


def gemv_naive(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """y = W x, bfloat16 W (m, n) and x (n,), binary32 y, in the naive tree: thread t sums
    a contiguous chunk of ceil(n / threads) columns, then a pairwise tree
    (src/pck/cuda/gemv.py:17-24; model `emulate_gemv`, src/pck/gemv.py:14-57)."""
    return extension().gemv_naive(W, x, threads)


def gemv_coalesced(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """y = W x in the coalesced tree (src/pck/cuda/gemv.py:27-34; model
    `emulate_gemv_coalesced(W, x, threads, 8)`, src/pck/gemv.py:71-101), ``threads`` a power
    of two in [32, 1024].

    ``x`` may also be a batch (B, n) with B <= 16: the result is then (B, m), every row
    bit-identical to the single-vector call on that column.
    """
    return extension().gemv_coalesced(W, x, threads)


def quantize_fp8(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(Q, s): E4M3 weights and binary32 per-row scales with W ~ s[:, None] * Q, s = max|w|
    / 448 per row, 1 for an all-zero row (src/pck/cuda/gemv.py:41-48). Weight-load time."""
    amax = W.abs().amax(dim=1).float()
    s = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    Q = (W.float() / s[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return Q.contiguous(), s


def gemv_fp8(Q: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """z = Q x for E4M3 ``Q`` (m, n) and bfloat16 ``x``: binary32 accumulation, 16 weights
    per 16-byte vector, bit-identical to `emulate_gemv_coalesced(Q, x, threads, 16)`
    (src/pck/cuda/gemv.py:51-58). The scales are applied by the caller: y = s * z."""
    return extension().gemv_fp8(Q, x, threads)
