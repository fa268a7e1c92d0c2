"""Trusted blocked checksum checker on the GPU (the drop-in for src/pck/cuda/checker.py).

The bank — secret signs r, binary32 checksums c = r^T W_beta and a_beta = sum |W_i|
rounded up to bfloat16 — is built at weight load: the signs are drawn from a CPU
torch.Generator exactly as the reference draws them (so the same generator state gives
the same r), and c, a are computed on the device by the library's bank kernel.

A check of y = W x, per check k and block beta of ``block`` rows:
    rho = c . x - r . y_beta,   tau = coef*s + geps*((1 + u32) s + sum |y_beta|) + tau_floor
with s an upper bound of a . |x|; a block passes iff its outputs are finite, tau is finite
and |rho| <= tau. The kernel evaluates rho in binary64 from exact products and every part
of tau rounded upward, so the reference's constants (coef, geps, tau_floor) bound its own
rounding with room to spare.

Modes:
  - `check` / `check_many`: the standalone check, a separate launch that reads y after
    the producing kernel finished (the reference's trust boundary);
  - `gemv_checked` / `checked_gemvs`: the GEMV and its check in ONE launch; each block's
    verdict is computed from y as stored, by the last unit of that block (production mode,
    non-adversarial faults).
A checker holds per-call scratch: use it from one stream at a time.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from dataclasses import dataclass

import torch

import pck.cuda.ops  # noqa: F401  (registers torch.ops.pck)
from pck.cuda import _lib
from pck.cuda._ext import MAX_BATCH, extension
from pck.fp import U32, U64, ceil_div, gamma, next_up, sum_up_factor

DEFAULT_BLOCK = 128
"""Rows per checksum."""

KERNEL_THREADS = 256  # the reference kernel's block size; enters its geps formula
BLOCKS_PER_SM = 4
MIN_SEGMENT_COLUMNS = 2 * KERNEL_THREADS


def round_up_bf16(v: torch.Tensor) -> torch.Tensor:
    """Non-negative binary64 values to bfloat16, never rounding down
    (src/pck/cuda/checker.py:29-43): up to binary32, then up to bfloat16 by carrying into
    bit 16 when any low bit is set. Past the range: +Inf."""
    if v.dtype != torch.float64:
        raise TypeError(f"round_up_bf16 expects float64, got {v.dtype}")
    if bool((v < 0).any()):
        raise ValueError("round_up_bf16 expects non-negative values")
    f = v.float()
    f = torch.where(f.double() < v, torch.nextafter(f, torch.full_like(f, math.inf)), f)
    bits = f.view(torch.int32)
    bits = torch.where((bits & 0xFFFF) != 0, (bits + 0x10000) & -0x10000, bits)
    return bits.view(torch.float32).to(torch.bfloat16)


@dataclass(frozen=True)
class CheckResult:
    """Per (check, block) outcome, each of shape (checks, num_blocks), or
    (batch, checks, num_blocks) for a batched check."""

    passed: torch.Tensor
    rho: torch.Tensor
    tau: torch.Tensor

    @property
    def verdict(self) -> torch.Tensor:
        """Per-block verdict: True only if the block passed every check."""
        return self.passed.all(dim=-2)


class GpuBlockedChecker:
    """Checks y = W x one block of ``block`` rows at a time with ``checks`` sign draws
    (src/pck/cuda/checker.py:61-129).

    ``height`` is the summation-tree height of the kernel being checked, e.g.
    `tree_height(n, threads, vec)`. ``segments`` splits every bank row into that many
    column segments (units of work); by default about four units per SM.
    """

    def __init__(self, W: torch.Tensor, block: int, height: int, checks: int = 1,
                 generator: torch.Generator | None = None, segments: int | None = None) -> None:  # fmt: skip
        if not (W.is_cuda and W.dtype == torch.bfloat16 and W.dim() == 2):
            raise ValueError("W must be a 2-D bfloat16 CUDA tensor")
        m, n = W.shape
        if block < 1 or m % block:
            raise ValueError(f"block={block} must be positive and divide m={m}")
        if checks < 1:
            raise ValueError(f"checks must be positive, got {checks}")
        self.m, self.n, self.block, self.checks = m, n, block, checks
        self.num_blocks = m // block
        self.height = height

        bits = torch.randint(0, 2, (checks, self.num_blocks, block), generator=generator)
        self.r = (2 * bits - 1).to(torch.int8).to(W.device)
        self.c, self.a = torch.ops.pck.bank_build(W.contiguous(), self.r, block, checks, sum_up_factor(block))
        if not bool(torch.isfinite(self.a).all()):
            raise ValueError("sum of |W| over a block overflows BF16")

        self.coef = next_up(gamma(height) + U32, 2)
        if segments is None:
            sms = torch.cuda.get_device_properties(W.device).multi_processor_count
            wanted = ceil_div(BLOCKS_PER_SM * sms, checks * self.num_blocks)
            segments = max(1, min(wanted, n // MIN_SEGMENT_COLUMNS))
        if not 1 <= segments <= min(n, 65535):
            raise ValueError(f"segments must be in [1, {min(n, 65535)}], got {segments}")
        self.segments = segments
        # The reference's geps (checker.py:320-329) covers a compensated binary32 dot product
        # per thread plus a binary64 reduction tree; the kernel here rounds less (binary64
        # from exact products), so the same constant bounds it.
        chain = ceil_div(ceil_div(n, segments), KERNEL_THREADS)
        g2 = gamma(2 * chain, U32) ** 2
        fp64_height = max(n + block + 1, 21 + segments + ceil_div(block, KERNEL_THREADS))
        gh = gamma(fp64_height, U64)
        self.geps = next_up(gh + g2 + gh * g2, 4)
        self.tau_floor = next_up(n * 2.0**-148, 2)
        self._scratch: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self._c64: torch.Tensor | None = None
        self._counters = torch.zeros((self.num_blocks,), dtype=torch.int32, device=W.device)
        self._partial_cx, self._partial_s = self.scratch(1)

    @property
    def c64(self) -> torch.Tensor:
        """c widened to binary64 (exact), made on first use: the tensor-core GEMV's fused
        reduction reads it instead of widening c in every stage."""
        if self._c64 is None:
            self._c64 = self.c.double()
        return self._c64

    def scratch(self, batch: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(partial_cx, partial_s) for a check of ``batch`` columns; batch 1 has no batch axis."""
        if batch not in self._scratch:
            lead = () if batch == 1 else (batch,)
            dev = self.c.device
            cx = torch.empty((*lead, self.checks, self.num_blocks, self.segments), dtype=torch.float64, device=dev)
            s = torch.empty((*lead, self.num_blocks, self.segments), dtype=torch.float64, device=dev)
            self._scratch[batch] = (cx, s)
        return self._scratch[batch]

    def check_args(self, x: torch.Tensor) -> tuple:
        """The bank, scratch and constants of a check of input ``x`` ((n,) or (B, n))."""
        batch = x.size(0) if x.dim() == 2 else 1
        pcx, ps = self.scratch(batch)
        return (self.c, self.a, self.r, pcx, ps, self._counters, self.coef, self.geps, self.tau_floor)

    def check(self, x: torch.Tensor, y: torch.Tensor) -> CheckResult:
        """Run every check on output ``y`` of the GEMV for input ``x``."""
        return check_many([(self, x, y)])[0]

    def verdict(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        """Per-block pass/fail (True = passed every check)."""
        return self.check(x, y).verdict


def check_many(items: Sequence[tuple[GpuBlockedChecker, torch.Tensor, torch.Tensor]]) -> list[CheckResult]:
    """Check several GEMV outputs ``(checker, x, y)``, up to 8 per launch
    (src/pck/cuda/checker.py:143-171). A checker may appear once per call."""
    if len({id(checker) for checker, _, _ in items}) != len(items):
        raise ValueError("each checker may appear only once per call")
    results: list[CheckResult] = []
    ext = extension()
    for i in range(0, len(items), MAX_BATCH):
        chunk = items[i : i + MAX_BATCH]
        args = [ch.check_args(x) for ch, x, _ in chunk]
        outputs = ext.blocked_check(
            [a[0] for a in args], [a[1] for a in args], [a[2] for a in args],
            [x for _, x, _ in chunk], [y for _, _, y in chunk],
            [a[3] for a in args], [a[4] for a in args], [a[5] for a in args],
            [a[6] for a in args], [a[7] for a in args], [a[8] for a in args],
        )  # fmt: skip
        results.extend(CheckResult(*out) for out in outputs)
    return results


def checked_gemvs(items: Sequence[tuple[torch.Tensor, torch.Tensor, GpuBlockedChecker | None]],
                  threads: int = 256) -> list[tuple[torch.Tensor, CheckResult | None]]:  # fmt: skip
    """Several GEMVs y = W x, each checked by its checker (or unchecked with None), in ONE
    persistent launch (up to 16): e.g. the projections of a decode layer that share their
    input. W may be bfloat16 or E4M3 (all items alike); x is (n,) or (B, n). Returns
    (y, CheckResult or None) per item. No reference counterpart: the reference launches
    every GEMV and the check separately."""
    if not items:
        return []
    if len({id(ch) for _, _, ch in items if ch is not None}) != sum(ch is not None for _, _, ch in items):
        raise ValueError("each checker may appear only once per call")
    W0 = items[0][0]
    fmt = _lib.PCK_WEIGHTS_E4M3 if W0.dtype == torch.float8_e4m3fn else _lib.PCK_WEIGHTS_BF16
    want = torch.float8_e4m3fn if fmt == _lib.PCK_WEIGHTS_E4M3 else torch.bfloat16
    jobs = []
    outs = []
    for W, x, ch in items:
        if not (W.is_cuda and x.is_cuda and W.device == W0.device and x.device == W0.device):
            raise RuntimeError("W and x must be CUDA tensors on one device")
        if W.dtype != want or x.dtype != torch.bfloat16:
            raise RuntimeError(f"W must be {want} (all items alike) and x bfloat16")
        if W.dim() != 2 or x.dim() not in (1, 2) or x.size(-1) != W.size(1):
            raise RuntimeError("expected W of shape (m, n) and x of shape (n,) or (B, n)")
        if not (W.is_contiguous() and x.is_contiguous()):
            raise RuntimeError("W and x must be contiguous")
        if ch is not None and (ch.m, ch.n) != tuple(W.shape):
            raise ValueError("the checker was built for another shape")
        y = torch.empty((*x.shape[:-1], W.size(0)), dtype=torch.float32, device=W.device)
        outs.append(y)
        jobs.append((W, x, y, None if ch is None else ch.check_args(x)))
    results: list[tuple[torch.Tensor, CheckResult | None]] = []
    ext = extension()
    for i in range(0, len(jobs), _lib.MAX_JOBS):
        part = jobs[i : i + _lib.MAX_JOBS]
        checks = ext.gemv_checked(part, threads, fmt)
        for (_, _, y, _), out in zip(part, checks, strict=True):
            results.append((y, None if out is None else CheckResult(*out)))
    return results


def gemv_checked(W: torch.Tensor, x: torch.Tensor, checker: GpuBlockedChecker,
                 threads: int = 256) -> tuple[torch.Tensor, CheckResult]:  # fmt: skip
    """y = W x and its check in one launch; returns (y, CheckResult)."""
    y, result = checked_gemvs([(W, x, checker)], threads)[0]
    assert result is not None
    return y, result


class PendingCheck:
    """A check queued on a side stream; `wait` makes the current stream wait for it
    (src/pck/cuda/checker.py:174-186)."""

    def __init__(self, result: CheckResult, done: torch.cuda.Event) -> None:
        self._result = result
        self._done = done

    def wait(self) -> CheckResult:
        stream = torch.cuda.current_stream()
        stream.wait_event(self._done)
        for t in (self._result.passed, self._result.rho, self._result.tau):
            t.record_stream(stream)
        return self._result


class SideStreamChecker:
    """Runs checks on a dedicated stream so they overlap later work
    (src/pck/cuda/checker.py:189-215). Each check starts after the work that produced y
    (an event recorded on the caller's stream at submit time); checks on one side stream
    run in order, so a checker's scratch is never shared by two checks in flight."""

    def __init__(self, device: torch.device | None = None) -> None:
        self.stream = torch.cuda.Stream(device)

    def submit(self, checker: GpuBlockedChecker, x: torch.Tensor, y: torch.Tensor) -> PendingCheck:
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            x.record_stream(self.stream)
            y.record_stream(self.stream)
            result = checker.check(x, y)
            done = torch.cuda.Event()
            done.record(self.stream)
        return PendingCheck(result, done)

    def wait_all(self) -> None:
        """Make the current stream wait for every check submitted so far."""
        torch.cuda.current_stream().wait_stream(self.stream)
