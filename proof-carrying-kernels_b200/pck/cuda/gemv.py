"""GEMV entry points (the GPU side of src/pck/cuda/gemv.py).

All of them run the sm_100a kernels of libpck_b200.so on the caller's current stream and
return binary32 outputs bit-identical to the reference's CPU models of its kernels.
"""

from __future__ import annotations

import torch

import pck.cuda.ops  # noqa: F401  (registers torch.ops.pck)

FP8_MAX = 448.0
"""Largest finite E4M3 value."""


def gemv_naive(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """y = W x, bfloat16 W (m, n) and x (n,), binary32 y, in the naive tree: thread t sums
    a contiguous chunk of ceil(n / threads) columns, then a pairwise tree
    (src/pck/cuda/gemv.py:17-24; model `emulate_gemv`, src/pck/gemv.py:14-57)."""
    return torch.ops.pck.gemv_naive(W, x, threads)


def gemv_coalesced(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    """y = W x in the coalesced tree (src/pck/cuda/gemv.py:27-34; model
    `emulate_gemv_coalesced(W, x, threads, 8)`, src/pck/gemv.py:71-101), ``threads`` a power
    of two in [32, 1024].

    ``x`` may also be a batch (B, n) with B <= 16: the result is then (B, m), every row
    bit-identical to the single-vector call on that column.
    """
    return torch.ops.pck.gemv_coalesced(W, x, threads)


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
    return torch.ops.pck.gemv_fp8(Q, x, threads)


TC_STEP_ROUNDINGS = 8
"""Roundings charged per tensor-core MMA step in `tc_height` (see there)."""


def tc_height(n: int) -> int:
    """Declared height of the tensor-core accumulation of `gemv_tc`, for its checker.

    Each tcgen05.mma adds 16 exact bfloat16 products to the binary32 accumulator, and the
    n / 16 MMAs of an output run in sequence. The hardware's internal rounding of one such
    step is not documented; this build assumes it is within ``TC_STEP_ROUNDINGS`` unit
    roundoffs of |accumulator| + sum |products| (published measurements of earlier tensor
    cores show at most 2 ulp of the largest addend, i.e. 4 u32, from truncating the
    aligned sum), so the whole chain is bounded by gamma_h with
    h = TC_STEP_ROUNDINGS * (ceil(n / 16) + 1). The GPU tests check every output against
    that bound and the checker for zero false alarms.
    """
    if n < 1:
        raise ValueError(f"n must be positive, got {n}")
    return TC_STEP_ROUNDINGS * (-(-n // 16) + 1)


def gemv_tc(W: torch.Tensor, X: torch.Tensor, checker=None, full_k: bool = False):
    """Y (B, m) = X (B, n) W^T on the tensor cores for a decode batch of 1 to 256 columns:
    bfloat16 or E4M3 W (m, n) and bfloat16 X (B, n), both contiguous and 16-byte aligned with
    n a multiple of 8 (16 for E4M3); binary32 Y. E4M3 weights are widened exactly to bfloat16
    in shared memory (their per-row scales are applied by the caller, y = s * z). Not
    bit-exact to the coalesced tree.

    With a ``checker`` (a GpuBlockedChecker of W, or of W widened to bfloat16 for E4M3 W,
    built with ``height=tc_height(n)``) the call also checks Y: the GEMV kernel reduces the
    bank rows against the staged X tiles in binary64 (128-row blocks, up to 2 checks, batches
    up to 128; other checkers take a bank launch of their own), a verdict launch decides the blocks, and the
    call returns (Y, CheckResult) with results of shape (B, checks, num_blocks).

    ``full_k``: every output accumulates its whole K range in one chain, so a row's value does
    not depend on the other rows of the call (row shards concatenate bit for bit to the
    unsharded result); otherwise a call of few row tiles may split K over a cluster of CTAs."""
    from pck.cuda.checker import CheckResult

    if checker is None:
        return torch.ops.pck.gemv_tc(W, X, full_k)
    if (checker.m, checker.n) != tuple(W.shape):
        raise ValueError("the checker was built for another shape")
    batch = X.size(0)
    pcx, ps = checker.scratch(batch)
    pcx = pcx.view(batch, checker.checks, checker.num_blocks, checker.segments)
    ps = ps.view(batch, checker.num_blocks, checker.segments)
    Y, passed, rho, tau = torch.ops.pck.gemv_tc_checked(W, X, checker.c, checker.a, checker.r, pcx, ps,
                                                        float(checker.coef), float(checker.geps),
                                                        float(checker.tau_floor), full_k, checker.c64)  # fmt: skip
    return Y, CheckResult(passed, rho, tau)
