"""Pre-validated launches for a decode loop: the tensors of a group of checked GEMVs are
fixed once, their C descriptors built once, and `launch()` issues the single
`pck_gemv_checked` call — cheap enough per token, and capturable in a CUDA graph.

`CheckedLayer` strings such launches into a transformer decode layer's projections
(q/k/v share an input, o, gate/up share an input, down), each group one persistent
launch with its checks fused.
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence

import torch

from pck.cuda import _lib
from pck.cuda._ext import extension, on_device, stream_handle
from pck.cuda.checker import CheckResult, GpuBlockedChecker


def exponent_range(W: torch.Tensor) -> tuple[int, int]:
    """(smallest exponent field of a nonzero weight, subnormals counted as 1; largest
    exponent field) of bfloat16 ``W``, or (0, 0) when W has no nonzero weight. With these
    the kernel can prove every product w*x exact in binary32 and add it with one FMA."""
    mag = W.view(torch.int16).to(torch.int32) & 0x7FFF
    exp = mag >> 7
    nonzero = mag != 0
    if not bool(nonzero.any()):
        return 0, 0
    lo = int(torch.where(nonzero, exp.clamp(min=1), torch.full_like(exp, 1000)).min())
    return lo, int(exp.max())


class GemvLaunch:
    """One launch of up to 16 GEMVs y_i = W_i x_i, each optionally checked.

    ``items``: (W, x, checker or None). W all bfloat16 or all E4M3, x (n,) or (B, n)
    bfloat16. ``ys`` may give preallocated outputs (e.g. views into one packed buffer);
    otherwise they are allocated. The results are rewritten by every launch.
    """

    def __init__(self, items: Sequence[tuple[torch.Tensor, torch.Tensor, GpuBlockedChecker | None]],
                 threads: int = 256, ys: Sequence[torch.Tensor] | None = None,
                 passed: Sequence[torch.Tensor | None] | None = None, verdicts: bool = True,
                 prior: Sequence[GemvLaunch] = ()) -> None:  # fmt: skip
        if not 1 <= len(items) <= _lib.MAX_JOBS:
            raise ValueError(f"a launch holds 1 to {_lib.MAX_JOBS} GEMVs, got {len(items)}")
        W0 = items[0][0]
        self.device = W0.device
        self.fmt = _lib.PCK_WEIGHTS_E4M3 if W0.dtype == torch.float8_e4m3fn else _lib.PCK_WEIGHTS_BF16
        want = torch.float8_e4m3fn if self.fmt == _lib.PCK_WEIGHTS_E4M3 else torch.bfloat16
        ext = extension()
        self.lib = ext.lib
        self.verdicts = verdicts
        self.count = len(items)
        self._descs = (_lib.CheckDesc * self.count)()
        self._jobs = (_lib.GemvJob * self.count)()
        self.items = list(items)
        self.ys: list[torch.Tensor] = []
        self.results: list[CheckResult | None] = []
        for g, (W, x, ch) in enumerate(items):
            if W.dtype != want or x.dtype != torch.bfloat16 or W.device != self.device or x.device != self.device:
                raise RuntimeError("W must share one format and device with the others, x bfloat16")
            if not (W.is_contiguous() and x.is_contiguous()) or x.size(-1) != W.size(1):
                raise RuntimeError("expected contiguous W (m, n) and x (n,) or (B, n)")
            shape = (*x.shape[:-1], W.size(0))
            y = ys[g] if ys is not None else torch.empty(shape, dtype=torch.float32, device=self.device)
            if tuple(y.shape) != shape or y.dtype != torch.float32 or not y.is_contiguous():
                raise RuntimeError(f"y must be a contiguous float32 tensor of shape {shape}")
            self.ys.append(y)
            job = self._jobs[g]
            job.W, job.X, job.Y = W.data_ptr(), x.data_ptr(), y.data_ptr()
            job.m, job.n = W.size(0), W.size(1)
            job.batch = x.size(0) if x.dim() == 2 else 1
            job.threads, job.weight_format = threads, self.fmt
            if self.fmt == _lib.PCK_WEIGHTS_BF16:
                job.w_exp_min, job.w_exp_max = exponent_range(W)
            if ch is None:
                job.check = None
                self.results.append(None)
                continue
            c, a, r, pcx, ps, ctr, coef, geps, floor = ch.check_args(x)
            out = ext.describe(c, a, r, x, y, pcx, ps, ctr, coef, geps, floor, self.device, self._descs[g])
            p = passed[g] if passed is not None else None
            if p is not None:  # write the verdict bits into the caller's buffer
                if p.numel() != out[0].numel() or p.dtype != torch.bool or not p.is_contiguous():
                    raise RuntimeError("passed must be a contiguous bool tensor of the check's size")
                self._descs[g].passed = p.data_ptr()
                out = (p.view(out[0].shape), out[1], out[2])
            self.results.append(CheckResult(*out))
            job.check = ctypes.pointer(self._descs[g])
        # The weights and the checkers' banks are final from here on (a launch object is made
        # at weight load), so the streaming kernel may request its first weight and bank pieces
        # before the preceding kernel on the stream has finished.
        torch.cuda.synchronize(self.device)
        for job in self._jobs:
            job.weight_format |= _lib.PCK_WEIGHTS_SETTLED
        for desc in self._descs:
            desc.flags |= _lib.PCK_CHECK_BANK_SETTLED
        self.prior: list[GemvLaunch] = []
        self._prior = None
        self.next: GemvLaunch | None = None
        self.set_prior(prior)

    def set_prior(self, launches: Sequence[GemvLaunch]) -> None:
        """Decide the checks of earlier launches (made with ``verdicts=False`` and launched
        before this one on the same stream) inside this launch (`pck_gemv_pipelined`): no
        verdict launch of their own. Their CheckResult objects then hold the verdicts once
        this launch has run."""
        descs = [d for gl in launches for d in gl.check_descs]
        if len(descs) > _lib.MAX_JOBS:
            raise ValueError(f"a launch decides at most {_lib.MAX_JOBS} prior checks, got {len(descs)}")
        if any(gl.verdicts for gl in launches):
            raise ValueError("prior launches must be made with verdicts=False")
        if descs and self.verdicts:
            raise ValueError("a launch that decides prior checks leaves its own to a later launch (verdicts=False)")
        self.prior = list(launches)  # keeps the checks' tensors alive
        self._prior = (_lib.CheckDesc * len(descs))(*descs) if descs else None

    def set_next(self, launch: GemvLaunch | None) -> None:
        """Name the launch that follows this one on the stream (``verdicts=False`` launches):
        this launch's CTAs then prefetch its first weight pieces into L2 as they finish
        (`pck_gemv_pipelined_next`). The results do not change."""
        if launch is not None and (self.verdicts or launch.device != self.device):
            raise ValueError("a next launch needs verdicts=False and the same device")
        self.next = launch

    def launch(self) -> None:
        """Issue the launch on the current stream (with ``verdicts=False``, the GEMVs and the
        checks' partial sums only; a VerdictLaunch, or a later launch given this one as
        ``prior``, decides the blocks)."""
        with on_device(self.device):
            stream = stream_handle(self.device)
            if self.verdicts:
                rc = self.lib.pck_gemv_checked(self._jobs, self.count, stream)
            elif self.next is not None:
                nprior = len(self._prior) if self._prior is not None else 0
                rc = self.lib.pck_gemv_pipelined_next(self._jobs, self.count, self._prior, nprior, self.next._jobs,
                                                      self.next.count, stream)  # fmt: skip
            elif self._prior is not None:
                rc = self.lib.pck_gemv_pipelined(self._jobs, self.count, self._prior, len(self._prior), stream)
            else:
                rc = self.lib.pck_gemv_partials(self._jobs, self.count, stream)
        _lib.check(rc, "checked gemv kernel")

    @property
    def check_descs(self) -> list:
        """The descriptors of this launch's checks (for a VerdictLaunch)."""
        return [self._descs[g] for g, res in enumerate(self.results) if res is not None]

    @property
    def algorithmic_bytes(self) -> int:
        """Bytes the launch must move at least: W, x, y and, for checked items, the bank
        (c, a, r) and the verdict outputs."""
        total = 0
        for (W, x, ch), y, res in zip(self.items, self.ys, self.results, strict=True):
            total += W.numel() * W.element_size() + x.numel() * 2 + y.numel() * 4
            if ch is not None:
                total += ch.c.numel() * 4 + ch.a.numel() * 2 + ch.r.numel()
                total += res.passed.numel() * (1 + 8 + 8)
        return total


class VerdictLaunch:
    """One launch of the verdict kernel for the checks of up to 16 GemvLaunch objects made
    with ``verdicts=False`` (e.g. every check of a decode layer, as the reference runs one
    checker launch per layer). Launch it on the same stream after them; their CheckResult
    objects then hold the verdicts."""

    def __init__(self, launches: Sequence[GemvLaunch]) -> None:
        descs = [d for gl in launches for d in gl.check_descs]
        if not 1 <= len(descs) <= _lib.MAX_JOBS:
            raise ValueError(f"a verdict launch covers 1 to {_lib.MAX_JOBS} checks, got {len(descs)}")
        self.launches = list(launches)  # keeps the checks' tensors alive
        self.device = launches[0].device
        self.lib = launches[0].lib
        self.count = len(descs)
        self._descs = (_lib.CheckDesc * self.count)(*descs)

    def launch(self) -> None:
        with on_device(self.device):
            rc = self.lib.pck_check_verdicts(self._descs, self.count, stream_handle(self.device))
        _lib.check(rc, "verdict kernel")


# Llama-3-8B decode-layer projections: (name, m, n) with hidden 4096, 8 KV heads of 128,
# MLP 14336; the groups share one input and form one launch each.
LLAMA3_8B_GROUPS: list[list[tuple[str, int, int]]] = [
    [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096)],
    [("o", 4096, 4096)],
    [("gate", 14336, 4096), ("up", 14336, 4096)],
    [("down", 4096, 14336)],
]


class TcLaunch:
    """One call of the tensor-core GEMV (`pck_gemv_tc`) for up to 8 matrices (all bfloat16 or
    all E4M3) that share a batch of activations, each optionally checked (a GpuBlockedChecker
    of W, widened to bfloat16 for E4M3, built with ``height=tc_height(n)``):
    Y_i (B, m_i) = X_i (B, n_i) W_i^T. Reusable launch after launch
    (e.g. captured in a CUDA graph); outputs in ``ys``, check results in ``results``."""

    def __init__(self, items: Sequence[tuple[torch.Tensor, torch.Tensor, GpuBlockedChecker | None]],
                 ys: Sequence[torch.Tensor] | None = None,
                 passed: Sequence[torch.Tensor | None] | None = None, full_k: bool = False) -> None:  # fmt: skip
        """``ys`` / ``passed`` may give preallocated outputs (e.g. views into the packed
        buffer of a row-sharded exchange): y (B, m) float32 and the verdict bits as a
        contiguous bool tensor of B * checks * num_blocks elements. ``full_k``: one
        accumulation chain over the whole K per output (`PCK_TC_FULL_K`), so row shards
        concatenate bit for bit to the unsharded result."""
        if not 1 <= len(items) <= 8:
            raise ValueError(f"a tensor-core launch holds 1 to 8 GEMVs, got {len(items)}")
        self.device = items[0][0].device
        self.lib = extension().lib
        self.count = len(items)
        self.items = list(items)
        self._descs = (_lib.CheckDesc * self.count)()
        self._jobs = (_lib.GemvJob * self.count)()
        self.ys: list[torch.Tensor] = []
        self.results: list[CheckResult | None] = []
        batch = items[0][1].size(0)
        wtype = items[0][0].dtype
        if wtype not in (torch.bfloat16, torch.float8_e4m3fn):
            raise RuntimeError("W must be bfloat16 or Float8_e4m3fn")
        fmt = _lib.PCK_WEIGHTS_E4M3 if wtype == torch.float8_e4m3fn else _lib.PCK_WEIGHTS_BF16
        for g, (W, X, ch) in enumerate(items):
            if W.dtype != wtype or X.dtype != torch.bfloat16 or X.dim() != 2 or X.size(0) != batch:
                raise RuntimeError("W must share one format, X be bfloat16 (B, n) with one B for the launch")
            if not (W.is_contiguous() and X.is_contiguous()) or X.size(1) != W.size(1):
                raise RuntimeError("expected contiguous W (m, n) and X (B, n)")
            shape = (batch, W.size(0))
            y = ys[g] if ys is not None else torch.empty(shape, dtype=torch.float32, device=self.device)
            if tuple(y.shape) != shape or y.dtype != torch.float32 or not y.is_contiguous():
                raise RuntimeError(f"y must be a contiguous float32 tensor of shape {shape}")
            self.ys.append(y)
            job = self._jobs[g]
            job.W, job.X, job.Y = W.data_ptr(), X.data_ptr(), y.data_ptr()
            job.m, job.n, job.batch, job.threads = W.size(0), W.size(1), batch, 256
            # the weights are final (synchronized below): the kernel may request its first
            # tiles while the kernel before it still runs
            job.weight_format = fmt | (_lib.PCK_TC_FULL_K if full_k else 0) | _lib.PCK_WEIGHTS_SETTLED
            if ch is None:
                job.check = None
                self.results.append(None)
                continue
            pcx, ps = ch.scratch(batch)
            shape = (batch, ch.checks, ch.num_blocks)
            p = passed[g] if passed is not None else None
            if p is not None and (p.numel() != math.prod(shape) or p.dtype != torch.bool or not p.is_contiguous()):
                raise RuntimeError("passed must be a contiguous bool tensor of the check's size")
            out = (p.view(shape) if p is not None else torch.empty(shape, dtype=torch.bool, device=self.device),
                   torch.empty(shape, dtype=torch.float64, device=self.device),
                   torch.empty(shape, dtype=torch.float64, device=self.device))  # fmt: skip
            d = self._descs[g]
            d.c, d.a, d.r, d.x, d.y = ch.c.data_ptr(), ch.a.data_ptr(), ch.r.data_ptr(), X.data_ptr(), y.data_ptr()
            d.partial_cx, d.partial_s, d.counters = pcx.data_ptr(), ps.data_ptr(), None
            d.passed, d.rho, d.tau = (t.data_ptr() for t in out)
            d.n, d.block, d.num_blocks, d.checks = W.size(1), ch.block, ch.num_blocks, ch.checks
            d.segments, d.batch = ch.segments, batch
            d.coef, d.geps, d.tau_floor = float(ch.coef), float(ch.geps), float(ch.tau_floor)
            d.c64 = ch.c64.data_ptr()
            job.check = ctypes.pointer(d)
            self.results.append(CheckResult(*out))
        torch.cuda.synchronize(self.device)

    def launch(self) -> None:
        with on_device(self.device):
            rc = self.lib.pck_gemv_tc(self._jobs, self.count, stream_handle(self.device))
        _lib.check(rc, "tensor-core gemv kernel")

    @property
    def algorithmic_bytes(self) -> int:
        """Bytes the launch must move at least: W, X and Y and, for checked items, the bank
        (c, a, r) and the verdict outputs (passed, rho, tau)."""
        total = 0
        for (W, X, ch), y, res in zip(self.items, self.ys, self.results, strict=True):
            total += W.numel() * W.element_size() + X.numel() * 2 + y.numel() * 4
            if ch is not None:
                total += ch.c.numel() * 4 + ch.a.numel() * 2 + ch.r.numel() + res.passed.numel() * (1 + 8 + 8)
        return total


class CapturedStep:
    """One decode step replayed from a CUDA graph, host buffers included: the copies of the
    step's inputs from pinned host memory, the step's launches (``body``, any sequence of the
    launch objects above plus collectives) and the copies of its results back to pinned host
    memory, captured once and replayed by `run` with a single graph launch. Refill the host
    input buffers between runs; `run` does not synchronize (read the host outputs after a
    `torch.cuda.synchronize()` or an event)."""

    def __init__(self, body, inputs: Sequence[tuple[torch.Tensor, torch.Tensor]],
                 outputs: Sequence[tuple[torch.Tensor, torch.Tensor]]) -> None:  # fmt: skip
        for host, dev in inputs:
            if not host.is_pinned() or host.shape != dev.shape or host.dtype != dev.dtype:
                raise ValueError("every input needs a pinned host buffer of the device tensor's shape and dtype")
        for dev, host in outputs:
            if not host.is_pinned() or host.shape != dev.shape or host.dtype != dev.dtype:
                raise ValueError("every output needs a pinned host buffer of the device tensor's shape and dtype")
        self.inputs, self.outputs = list(inputs), list(outputs)

        def step() -> None:
            for host, dev in self.inputs:
                dev.copy_(host, non_blocking=True)
            body()
            for dev, host in self.outputs:
                host.copy_(dev, non_blocking=True)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()  # once eagerly (lazy initialisation stays out of the graph)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            step()
        torch.cuda.synchronize()

    @property
    def h2d_bytes(self) -> int:
        return sum(h.numel() * h.element_size() for h, _ in self.inputs)

    @property
    def d2h_bytes(self) -> int:
        return sum(h.numel() * h.element_size() for _, h in self.outputs)

    def run(self) -> None:
        self.graph.replay()
