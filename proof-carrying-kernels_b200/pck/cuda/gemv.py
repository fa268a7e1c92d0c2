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


def gemv_tc(W: torch.Tensor, X: torch.Tensor, checker=None):
    """Y (B, m) = X (B, n) W^T on the tensor cores for a decode batch of 1 to 256 columns:
    bfloat16 W (m, n) and X (B, n), both contiguous and 16-byte aligned with n a multiple of
    8; binary32 Y. Not bit-exact to the coalesced tree.

    With a ``checker`` (a GpuBlockedChecker of W built with ``height=tc_height(n)``) the
    call also checks Y: a binary64 launch reduces the bank rows against X (every batch
    column), a verdict launch decides the blocks, and the call returns (Y, CheckResult) with
    results of shape (B, checks, num_blocks)."""
    import ctypes

    from pck.cuda import _lib
    from pck.cuda._ext import check_cuda, on_device, ptr, stream_handle
    from pck.cuda.checker import CheckResult

    if not (W.is_cuda and X.is_cuda and W.device == X.device):
        raise RuntimeError("W and X must be CUDA tensors on one device")
    if W.dtype != torch.bfloat16 or X.dtype != torch.bfloat16:
        raise RuntimeError("W and X must be bfloat16")
    if W.dim() != 2 or X.dim() != 2 or X.size(1) != W.size(1):
        raise RuntimeError("expected W of shape (m, n) and X of shape (B, n)")
    if not (W.is_contiguous() and X.is_contiguous()):
        raise RuntimeError("W and X must be contiguous")
    batch = X.size(0)
    dev = W.device
    Y = torch.empty((batch, W.size(0)), dtype=torch.float32, device=dev)
    job = (_lib.GemvJob * 1)()
    job[0].W, job[0].X, job[0].Y = W.data_ptr(), X.data_ptr(), Y.data_ptr()
    job[0].m, job[0].n, job[0].batch, job[0].threads = W.size(0), W.size(1), batch, 256
    job[0].weight_format = _lib.PCK_WEIGHTS_BF16
    job[0].check = ctypes.POINTER(_lib.CheckDesc)()
    result = None
    desc = _lib.CheckDesc()
    if checker is not None:
        if (checker.m, checker.n) != tuple(W.shape):
            raise ValueError("the checker was built for another shape")
        pcx, ps = checker.scratch(batch)
        pcx = pcx.view(batch, checker.checks, checker.num_blocks, checker.segments)
        ps = ps.view(batch, checker.num_blocks, checker.segments)
        for t, name, dt in ((pcx, "partial_cx", torch.float64), (ps, "partial_s", torch.float64)):
            check_cuda(t, name, dt, dev)
        shape = (batch, checker.checks, checker.num_blocks)
        passed = torch.empty(shape, dtype=torch.bool, device=dev)
        rho = torch.empty(shape, dtype=torch.float64, device=dev)
        tau = torch.empty(shape, dtype=torch.float64, device=dev)
        desc.c, desc.a, desc.r = ptr(checker.c), ptr(checker.a), ptr(checker.r)
        desc.x, desc.y = ptr(X), ptr(Y)
        desc.partial_cx, desc.partial_s, desc.counters = ptr(pcx), ptr(ps), None
        desc.passed, desc.rho, desc.tau = ptr(passed), ptr(rho), ptr(tau)
        desc.n, desc.block, desc.num_blocks, desc.checks = W.size(1), checker.block, checker.num_blocks, checker.checks
        desc.segments, desc.batch = checker.segments, batch
        desc.coef, desc.geps, desc.tau_floor = float(checker.coef), float(checker.geps), float(checker.tau_floor)
        job[0].check = ctypes.pointer(desc)
        result = CheckResult(passed, rho, tau)
    with on_device(dev):
        rc = _lib.library().pck_gemv_tc(job, 1, stream_handle(dev))
    _lib.check(rc, "tensor-core gemv kernel")
    return Y if checker is None else (Y, result)
