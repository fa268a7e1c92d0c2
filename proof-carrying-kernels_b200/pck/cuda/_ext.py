"""Tensor-level wrappers of the C ABI, mirroring the reference's pybind11 module
`pck_kernels` (src/pck/cuda/csrc/bindings.cpp:302-335): same function names, argument
order, validation order and error wording (RuntimeError, as TORCH_CHECK raises).

`extension()` returns the wrapper object; `pck.cuda` builds the public API on it.
"""

from __future__ import annotations

import contextlib
import ctypes
import functools
from collections.abc import Sequence

import torch

from pck.cuda import _lib

INT32_MAX = 2**31 - 1
MAX_BATCH = 8  # checks per `blocked_check` call, as the reference's kMaxBatch (checker.h:36)

_TYPE_NAMES = {
    torch.float32: "Float",
    torch.float64: "Double",
    torch.bfloat16: "BFloat16",
    torch.float16: "Half",
    torch.int8: "Char",
    torch.uint8: "Byte",
    torch.int32: "Int",
    torch.int64: "Long",
    torch.bool: "Bool",
    torch.float8_e4m3fn: "Float8_e4m3fn",
}


def type_name(dtype: torch.dtype) -> str:
    return _TYPE_NAMES.get(dtype, str(dtype).removeprefix("torch."))


def on_device(device: torch.device):
    """Makes ``device`` current for the duration (the C ABI launches on the current device)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def check_cuda(t: torch.Tensor, name: str, dtype: torch.dtype, device: torch.device) -> None:
    """bindings.cpp:154-159."""
    if not (t.is_cuda and t.device == device):
        raise RuntimeError(f"{name} must be on {device}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {type_name(dtype)}, got {type_name(t.dtype)}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


class Extension:
    """The entry points of the CUDA library on torch tensors."""

    def __init__(self) -> None:
        self.lib = _lib.library()

    # -- GEMV (bindings.cpp:45-83) -----------------------------------------------------
    def _gemv(self, W: torch.Tensor, x: torch.Tensor, threads: int, min_threads: int,
              w_type: torch.dtype, weight_format: int, naive: bool = False) -> torch.Tensor:  # fmt: skip
        if not (W.is_cuda and x.is_cuda):
            raise RuntimeError("W and x must be CUDA tensors")
        if W.device != x.device:
            raise RuntimeError("W and x must be on the same device")
        if W.dtype != w_type or x.dtype != torch.bfloat16:
            raise RuntimeError(f"W must be {type_name(w_type)} and x bfloat16")
        batched = x.dim() == 2 and not naive
        if not (W.dim() == 2 and (x.dim() == 1 or batched) and x.size(-1) == W.size(1)):
            want = "(n,) or (B, n)" if not naive else "(n,)"
            raise RuntimeError(
                f"expected W of shape (m, n) and x of shape {want}, got {list(W.shape)} and {list(x.shape)}"
            )
        if not (W.is_contiguous() and x.is_contiguous()):
            raise RuntimeError("W and x must be contiguous")
        if not (min_threads <= threads <= 1024 and threads & (threads - 1) == 0):
            raise RuntimeError(f"threads must be a power of two in [{min_threads}, 1024], got {threads}")
        if W.size(0) > INT32_MAX:
            raise RuntimeError("too many rows")
        m, n = W.shape
        batch = x.size(0) if batched else 1
        if batched and not 1 <= batch <= _lib.MAX_BATCH:
            raise RuntimeError(f"batch size must be in [1, {_lib.MAX_BATCH}], got {batch}")
        y = torch.empty((batch, m) if batched else (m,), dtype=torch.float32, device=W.device)
        if m == 0:
            return y
        if n <= 0:
            raise RuntimeError("n must be positive")
        with on_device(W.device):
            s = stream_handle(W.device)
            if naive:
                rc = self.lib.pck_gemv_naive(ptr(W), ptr(x), ptr(y), m, n, threads, s)
            else:
                rc = self.lib.pck_gemv_batched(weight_format, ptr(W), ptr(x), ptr(y), m, n, batch,
                                               threads, s)  # fmt: skip
        _lib.check(rc, "gemv kernel")
        return y

    def gemv_naive(self, W: torch.Tensor, x: torch.Tensor, threads: int) -> torch.Tensor:
        return self._gemv(W, x, threads, 1, torch.bfloat16, _lib.PCK_WEIGHTS_BF16, naive=True)

    def gemv_coalesced(self, W: torch.Tensor, x: torch.Tensor, threads: int) -> torch.Tensor:
        return self._gemv(W, x, threads, 32, torch.bfloat16, _lib.PCK_WEIGHTS_BF16)

    def gemv_fp8(self, Q: torch.Tensor, x: torch.Tensor, threads: int) -> torch.Tensor:
        return self._gemv(Q, x, threads, 32, torch.float8_e4m3fn, _lib.PCK_WEIGHTS_E4M3)

    # -- blocked checker (bindings.cpp:161-256) ----------------------------------------
    def describe(self, c, a, r, x, y, partial_cx, partial_s, counters, coef: float, geps: float,
                 tau_floor: float, device: torch.device, d: _lib.CheckDesc):  # fmt: skip
        """Validates one check and fills its descriptor; returns its output tensors."""
        check_cuda(c, "c", torch.float32, device)
        check_cuda(a, "a", torch.bfloat16, device)
        check_cuda(r, "r", torch.int8, device)
        check_cuda(x, "x", torch.bfloat16, device)
        check_cuda(y, "y", torch.float32, device)
        check_cuda(partial_cx, "partial_cx", torch.float64, device)
        check_cuda(partial_s, "partial_s", torch.float64, device)
        check_cuda(counters, "counters", torch.int32, device)
        if not (c.dim() == 3 and a.dim() == 2 and r.dim() == 3 and x.dim() in (1, 2) and y.dim() == x.dim()):
            raise RuntimeError("expected c (K, nb, n), a (nb, n), r (K, nb, b), x (n,), y (m,)")
        checks, num_blocks, n = c.shape
        block = r.size(2)
        batch = x.size(0) if x.dim() == 2 else 1
        if a.shape != (num_blocks, n):
            raise RuntimeError("a must have shape (nb, n)")
        if r.size(0) != checks or r.size(1) != num_blocks:
            raise RuntimeError("r must have shape (K, nb, b)")
        if x.size(-1) != n:
            raise RuntimeError("x must have shape (n,)")
        if y.size(-1) != num_blocks * block or (x.dim() == 2 and y.size(0) != batch):
            raise RuntimeError("y must have shape (nb * b,)")
        if not (checks >= 1 and num_blocks >= 1 and n >= 1 and block >= 1):
            raise RuntimeError("empty checker")
        if not 1 <= batch <= _lib.MAX_BATCH:
            raise RuntimeError(f"batch size must be in [1, {_lib.MAX_BATCH}], got {batch}")
        lead = (batch,) if x.dim() == 2 else ()
        if partial_cx.dim() != len(lead) + 3 or tuple(partial_cx.shape[:-1]) != (*lead, checks, num_blocks):
            raise RuntimeError("partial sums must have shape (K, nb, segments)")
        segments = partial_cx.size(-1)
        if tuple(partial_s.shape) != (*lead, num_blocks, segments):
            raise RuntimeError("partial sums must have shape (K, nb, segments)")
        if tuple(counters.shape) != (num_blocks,):
            raise RuntimeError("counters must have shape (nb,)")
        if not 1 <= segments <= n:
            raise RuntimeError(f"segments must be in [1, n], got {segments}")
        if not (coef > 0 and geps > 0 and tau_floor > 0):
            raise RuntimeError("coef, geps and floor must be positive")
        shape = (*lead, checks, num_blocks)
        passed = torch.empty(shape, dtype=torch.bool, device=device)
        rho = torch.empty(shape, dtype=torch.float64, device=device)
        tau = torch.empty(shape, dtype=torch.float64, device=device)
        d.c, d.a, d.r, d.x, d.y = ptr(c), ptr(a), ptr(r), ptr(x), ptr(y)
        d.partial_cx, d.partial_s, d.counters = ptr(partial_cx), ptr(partial_s), ptr(counters)
        d.passed, d.rho, d.tau = ptr(passed), ptr(rho), ptr(tau)
        d.n, d.block, d.num_blocks, d.checks = n, block, num_blocks, checks
        d.segments, d.batch = segments, batch
        d.coef, d.geps, d.tau_floor = float(coef), float(geps), float(tau_floor)
        return passed, rho, tau

    def blocked_check(self, c: Sequence[torch.Tensor], a, r, x, y, partial_cx, partial_s,
                      counters, coef, geps, tau_floor) -> list:  # fmt: skip
        """Up to 8 checks in one launch; (passed, rho, tau) per check."""
        count = len(c)
        if not 1 <= count <= MAX_BATCH:
            raise RuntimeError(f"batch size must be in [1, {MAX_BATCH}], got {count}")
        lists = (a, r, x, y, partial_cx, partial_s, counters, coef, geps, tau_floor)
        if any(len(v) != count for v in lists):
            raise RuntimeError("all argument lists must have the same length")
        if not y[0].is_cuda:
            raise RuntimeError("y must be a CUDA tensor")
        device = y[0].device
        descs = (_lib.CheckDesc * count)()
        outputs = []
        for g in range(count):
            if not y[g].is_cuda:
                raise RuntimeError("y must be a CUDA tensor")
            outputs.append(self.describe(c[g], a[g], r[g], x[g], y[g], partial_cx[g], partial_s[g],
                                         counters[g], coef[g], geps[g], tau_floor[g], device,
                                         descs[g]))  # fmt: skip
        with on_device(device):
            rc = self.lib.pck_blocked_check(descs, count, stream_handle(device))
        _lib.check(rc, "checker kernel")
        return outputs

    # -- fused checked GEMVs (no reference counterpart) --------------------------------
    def gemv_checked(self, jobs: Sequence[tuple], threads: int, weight_format: int) -> list:
        """jobs: (W, x, y, check_args or None) with check_args the `describe` arguments
        after x and y. One launch; returns the outputs of each check (or None)."""
        count = len(jobs)
        if not 1 <= count <= _lib.MAX_JOBS:
            raise RuntimeError(f"batch size must be in [1, {_lib.MAX_JOBS}], got {count}")
        device = jobs[0][0].device
        descs = (_lib.CheckDesc * count)()
        arr = (_lib.GemvJob * count)()
        outputs = []
        for g, (W, x, y, chk) in enumerate(jobs):
            batch = x.size(0) if x.dim() == 2 else 1
            job = arr[g]
            job.W, job.X, job.Y = ptr(W), ptr(x), ptr(y)
            job.m, job.n = W.size(0), W.size(1)
            job.batch, job.threads, job.weight_format = batch, threads, weight_format
            if chk is None:
                job.check = None
                outputs.append(None)
            else:
                c, a, r, pcx, ps, ctr, coef, geps, floor = chk
                outputs.append(self.describe(c, a, r, x, y, pcx, ps, ctr, coef, geps, floor, device,
                                             descs[g]))  # fmt: skip
                job.check = ctypes.pointer(descs[g])
        with on_device(device):
            rc = self.lib.pck_gemv_checked(arr, count, stream_handle(device))
        _lib.check(rc, "checked gemv kernel")
        return outputs

    # -- bank at weight load -----------------------------------------------------------
    def bank_build(self, W: torch.Tensor, r: torch.Tensor, c: torch.Tensor, a: torch.Tensor,
                   block: int, checks: int, factor: float) -> None:  # fmt: skip
        m, n = W.shape
        with on_device(W.device):
            rc = self.lib.pck_bank_build(ptr(W), ptr(r), ptr(c), ptr(a), m, n, block, checks,
                                         float(factor), stream_handle(W.device))  # fmt: skip
        _lib.check(rc, "bank kernel")


@functools.cache
def extension() -> Extension:
    """The loaded CUDA library (raises RuntimeError if it is not built)."""
    return Extension()
