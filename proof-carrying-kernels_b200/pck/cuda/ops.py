"""The library's entry points as PyTorch custom operators (namespace ``pck``), the drop-in for
the reference's extension module `pck_kernels` (src/pck/cuda/csrc/bindings.cpp:302-335): the
same operations reach the dispatcher, so `torch.compile`, `make_fx` and fake-tensor tracing
see them as single opaque nodes, with fake (meta) implementations that give every output's
shape and dtype without running a kernel. Each real implementation is one call of the C ABI
(include/pck_b200.h) through `pck.cuda._ext`, on the current stream; it validates its
arguments first with the reference's error wording (CPU tensors are rejected there, as the
reference rejects them, rather than by a missing dispatch key).

    torch.ops.pck.gemv_naive(W, x, threads)           -> y
    torch.ops.pck.gemv_coalesced(W, x, threads)       -> y       (x (n,) or (B, n), B <= 16)
    torch.ops.pck.gemv_fp8(Q, x, threads)             -> z
    torch.ops.pck.gemv_tc(W, X, full_k=False)         -> Y       (B <= 256, bfloat16 or E4M3 W)
    torch.ops.pck.blocked_check(c, a, r, x, y, partial_cx!, partial_s!, coef, geps, tau_floor)
                                                      -> (passed, rho, tau)
    torch.ops.pck.gemv_checked(W, x, c, a, r, partial_cx!, partial_s!, coef, geps, tau_floor, threads)
                                                      -> (y, passed, rho, tau)
    torch.ops.pck.gemv_tc_checked(W, X, c, a, r, partial_cx!, partial_s!, coef, geps, tau_floor, full_k=False,
                                  c64=None)
                                                      -> (Y, passed, rho, tau)
    torch.ops.pck.member_check(logits, tokens, top_k?, top_p?, greedy?, slack) -> (ok, above, mass_above)
    torch.ops.pck.sampling_check(logits, selected, lengths, k, top_p, p, temperature, slack, segments)
                                                      -> (passed, min_selected, max_rejected, mass, without)
    torch.ops.pck.bank_build(W, r, block, checks, factor) -> (c, a)

``!`` marks the checks' scratch (binary64 partial sums), which the operators write.
"""

from __future__ import annotations

import ctypes

import torch

from pck.cuda import _lib

_FLOAT = torch.float32


def _ext():
    from pck.cuda._ext import extension

    return extension()


def _check_outputs(x: torch.Tensor, c: torch.Tensor) -> tuple[int, ...]:
    """(…, checks, num_blocks): the shape of a check's outputs for activations x."""
    lead = (x.size(0),) if x.dim() == 2 else ()
    return (*lead, c.size(0), c.size(1))


# -- GEMV ------------------------------------------------------------------------------


@torch.library.custom_op("pck::gemv_naive", mutates_args=())
def gemv_naive(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    return _ext().gemv_naive(W, x, threads)


@gemv_naive.register_fake
def _(W, x, threads=256):
    return W.new_empty((W.size(0),), dtype=_FLOAT)


@torch.library.custom_op("pck::gemv_coalesced", mutates_args=())
def gemv_coalesced(W: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    return _ext().gemv_coalesced(W, x, threads)


@gemv_coalesced.register_fake
def _(W, x, threads=256):
    return W.new_empty((*x.shape[:-1], W.size(0)), dtype=_FLOAT)


@torch.library.custom_op("pck::gemv_fp8", mutates_args=())
def gemv_fp8(Q: torch.Tensor, x: torch.Tensor, threads: int = 256) -> torch.Tensor:
    return _ext().gemv_fp8(Q, x, threads)


@gemv_fp8.register_fake
def _(Q, x, threads=256):
    return Q.new_empty((*x.shape[:-1], Q.size(0)), dtype=_FLOAT)


def _tc_job(W: torch.Tensor, X: torch.Tensor, Y: torch.Tensor, full_k: bool = False):
    if not (W.is_cuda and X.is_cuda and W.device == X.device):
        raise RuntimeError("W and X must be CUDA tensors on one device")
    if W.dtype not in (torch.bfloat16, torch.float8_e4m3fn) or X.dtype != torch.bfloat16:
        raise RuntimeError("W must be bfloat16 or Float8_e4m3fn and X bfloat16")
    if W.dim() != 2 or X.dim() != 2 or X.size(1) != W.size(1):
        raise RuntimeError("expected W of shape (m, n) and X of shape (B, n)")
    if not (W.is_contiguous() and X.is_contiguous()):
        raise RuntimeError("W and X must be contiguous")
    job = (_lib.GemvJob * 1)()
    job[0].W, job[0].X, job[0].Y = W.data_ptr(), X.data_ptr(), Y.data_ptr()
    job[0].m, job[0].n, job[0].batch, job[0].threads = W.size(0), W.size(1), X.size(0), 256
    job[0].weight_format = _lib.PCK_WEIGHTS_E4M3 if W.dtype == torch.float8_e4m3fn else _lib.PCK_WEIGHTS_BF16
    if full_k:
        job[0].weight_format |= _lib.PCK_TC_FULL_K
    job[0].check = ctypes.POINTER(_lib.CheckDesc)()
    return job


def _run_tc(job, device: torch.device) -> None:
    from pck.cuda._ext import on_device, stream_handle

    with on_device(device):
        rc = _lib.library().pck_gemv_tc(job, 1, stream_handle(device))
    _lib.check(rc, "tensor-core gemv kernel")


@torch.library.custom_op("pck::gemv_tc", mutates_args=())
def gemv_tc(W: torch.Tensor, X: torch.Tensor, full_k: bool = False) -> torch.Tensor:
    Y = torch.empty((X.size(0), W.size(0)), dtype=_FLOAT, device=W.device)
    _run_tc(_tc_job(W, X, Y, full_k), W.device)
    return Y


@gemv_tc.register_fake
def _(W, X, full_k=False):
    return X.new_empty((X.size(0), W.size(0)), dtype=_FLOAT)


# -- checks ----------------------------------------------------------------------------


@torch.library.custom_op("pck::blocked_check", mutates_args=("partial_cx", "partial_s"))
def blocked_check(c: torch.Tensor, a: torch.Tensor, r: torch.Tensor, x: torch.Tensor, y: torch.Tensor,
                  partial_cx: torch.Tensor, partial_s: torch.Tensor, coef: float, geps: float,
                  tau_floor: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    counters = torch.empty((c.size(1),), dtype=torch.int32, device=y.device)
    (out,) = _ext().blocked_check([c], [a], [r], [x], [y], [partial_cx], [partial_s], [counters], [coef], [geps],
                                  [tau_floor])  # fmt: skip
    return out


@blocked_check.register_fake
def _(c, a, r, x, y, partial_cx, partial_s, coef, geps, tau_floor):
    shape = _check_outputs(x, c)
    return (y.new_empty(shape, dtype=torch.bool), y.new_empty(shape, dtype=torch.float64),
            y.new_empty(shape, dtype=torch.float64))  # fmt: skip


@torch.library.custom_op("pck::gemv_checked", mutates_args=("partial_cx", "partial_s"))
def gemv_checked(W: torch.Tensor, x: torch.Tensor, c: torch.Tensor, a: torch.Tensor, r: torch.Tensor,
                 partial_cx: torch.Tensor, partial_s: torch.Tensor, coef: float, geps: float, tau_floor: float,
                 threads: int = 256) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    fmt = _lib.PCK_WEIGHTS_E4M3 if W.dtype == torch.float8_e4m3fn else _lib.PCK_WEIGHTS_BF16
    y = torch.empty((*x.shape[:-1], W.size(0)), dtype=_FLOAT, device=W.device)
    counters = torch.empty((c.size(1),), dtype=torch.int32, device=W.device)
    (out,) = _ext().gemv_checked([(W, x, y, (c, a, r, partial_cx, partial_s, counters, coef, geps, tau_floor))],
                                 threads, fmt)  # fmt: skip
    return (y, *out)


@gemv_checked.register_fake
def _(W, x, c, a, r, partial_cx, partial_s, coef, geps, tau_floor, threads=256):
    shape = _check_outputs(x, c)
    return (W.new_empty((*x.shape[:-1], W.size(0)), dtype=_FLOAT), W.new_empty(shape, dtype=torch.bool),
            W.new_empty(shape, dtype=torch.float64), W.new_empty(shape, dtype=torch.float64))  # fmt: skip


@torch.library.custom_op("pck::gemv_tc_checked", mutates_args=("partial_cx", "partial_s"))
def gemv_tc_checked(W: torch.Tensor, X: torch.Tensor, c: torch.Tensor, a: torch.Tensor, r: torch.Tensor,
                    partial_cx: torch.Tensor, partial_s: torch.Tensor, coef: float, geps: float,
                    tau_floor: float, full_k: bool = False,
                    c64: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    Y = torch.empty((X.size(0), W.size(0)), dtype=_FLOAT, device=W.device)
    job = _tc_job(W, X, Y, full_k)
    desc = _lib.CheckDesc()
    batch = X.size(0)
    shape = (batch, c.size(0), c.size(1))
    if tuple(partial_cx.shape[:-1]) != shape or tuple(partial_s.shape[:-1]) != (batch, c.size(1)):
        raise RuntimeError("partial sums must have shape (B, K, nb, segments) and (B, nb, segments)")
    passed = torch.empty(shape, dtype=torch.bool, device=W.device)
    rho = torch.empty(shape, dtype=torch.float64, device=W.device)
    tau = torch.empty(shape, dtype=torch.float64, device=W.device)
    desc.c, desc.a, desc.r, desc.x, desc.y = c.data_ptr(), a.data_ptr(), r.data_ptr(), X.data_ptr(), Y.data_ptr()
    desc.partial_cx, desc.partial_s, desc.counters = partial_cx.data_ptr(), partial_s.data_ptr(), None
    desc.passed, desc.rho, desc.tau = passed.data_ptr(), rho.data_ptr(), tau.data_ptr()
    desc.n, desc.block, desc.num_blocks, desc.checks = W.size(1), r.size(2), c.size(1), c.size(0)
    desc.segments, desc.batch = partial_cx.size(-1), batch
    desc.coef, desc.geps, desc.tau_floor = float(coef), float(geps), float(tau_floor)
    if c64 is not None:
        if c64.dtype != torch.float64 or c64.shape != c.shape or not c64.is_contiguous() or c64.device != c.device:
            raise RuntimeError("c64 must be a contiguous float64 tensor of c's shape and device")
        desc.c64 = c64.data_ptr()
    job[0].check = ctypes.pointer(desc)
    _run_tc(job, W.device)
    return Y, passed, rho, tau


@gemv_tc_checked.register_fake
def _(W, X, c, a, r, partial_cx, partial_s, coef, geps, tau_floor, full_k=False, c64=None):
    shape = (X.size(0), c.size(0), c.size(1))
    return (X.new_empty((X.size(0), W.size(0)), dtype=_FLOAT), X.new_empty(shape, dtype=torch.bool),
            X.new_empty(shape, dtype=torch.float64), X.new_empty(shape, dtype=torch.float64))  # fmt: skip


# -- membership and set checks ---------------------------------------------------------

_LOGITS = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}  # PCK_LOGITS_*


@torch.library.custom_op("pck::member_check", mutates_args=())
def member_check(logits: torch.Tensor, tokens: torch.Tensor, top_k: torch.Tensor | None, top_p: torch.Tensor | None,
                 greedy: torch.Tensor | None, slack: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    from pck.cuda._ext import on_device, stream_handle

    if logits.dim() != 2 or logits.dtype not in _LOGITS or logits.stride(1) != 1:
        raise RuntimeError("logits must be (B, V) float32, bfloat16 or float16 with unit column stride")
    rows, vocab = logits.shape
    dev = logits.device
    for t, name, dt in ((tokens, "tokens", torch.int64), (top_k, "top_k", torch.int64),
                        (top_p, "top_p", torch.float64), (greedy, "greedy", torch.bool)):  # fmt: skip
        if t is not None and (t.dtype != dt or t.numel() != rows or not t.is_contiguous() or t.device != dev):
            raise RuntimeError(f"{name} must be a contiguous {dt} tensor of one value per row on {dev}")
    ok = torch.empty(rows, dtype=torch.bool, device=dev)
    above = torch.empty(rows, dtype=torch.int64, device=dev)
    mass = torch.empty(rows, dtype=torch.float64, device=dev)

    def p(t):
        return None if t is None else t.data_ptr()

    with on_device(dev):
        rc = _lib.library().pck_member_check(logits.data_ptr(), _LOGITS[logits.dtype], rows, vocab, logits.stride(0),
                                             tokens.data_ptr(), p(top_k), p(top_p), p(greedy), slack, ok.data_ptr(),
                                             above.data_ptr(), mass.data_ptr(), stream_handle(dev))  # fmt: skip
    _lib.check(rc, "membership kernel")
    return ok, above, mass


@member_check.register_fake
def _(logits, tokens, top_k, top_p, greedy, slack):
    rows = logits.size(0)
    return (logits.new_empty((rows,), dtype=torch.bool), logits.new_empty((rows,), dtype=torch.int64),
            logits.new_empty((rows,), dtype=torch.float64))  # fmt: skip


@torch.library.custom_op("pck::sampling_check", mutates_args=())
def sampling_check(logits: torch.Tensor, selected: torch.Tensor, lengths: torch.Tensor, k: int, top_p: bool,
                   p: float, temperature: float, slack: float, segments: int
                   ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:  # fmt: skip
    from pck.cuda.sampling import _run

    out = _run(logits, selected, lengths, k, top_p, p, temperature, slack, segments)
    return out.passed, out.min_selected, out.max_rejected, out.mass, out.mass_without_smallest


@sampling_check.register_fake
def _(logits, selected, lengths, k, top_p, p, temperature, slack, segments):
    rows = logits.size(0)
    return (logits.new_empty((rows,), dtype=torch.bool), logits.new_empty((rows,), dtype=torch.float32),
            logits.new_empty((rows,), dtype=torch.float32), logits.new_empty((rows,), dtype=torch.float64),
            logits.new_empty((rows,), dtype=torch.float64))  # fmt: skip


# -- bank at weight load ---------------------------------------------------------------


@torch.library.custom_op("pck::bank_build", mutates_args=())
def bank_build(W: torch.Tensor, r: torch.Tensor, block: int, checks: int,
               factor: float) -> tuple[torch.Tensor, torch.Tensor]:  # fmt: skip
    m, n = W.shape
    c = torch.empty((checks, m // block, n), dtype=torch.float32, device=W.device)
    a = torch.empty((m // block, n), dtype=torch.bfloat16, device=W.device)
    _ext().bank_build(W.contiguous(), r.contiguous(), c, a, block, checks, factor)
    return c, a


@bank_build.register_fake
def _(W, r, block, checks, factor):
    m, n = W.shape
    return (W.new_empty((checks, m // block, n), dtype=torch.float32),
            W.new_empty((m // block, n), dtype=torch.bfloat16))  # fmt: skip


OPS = ("gemv_naive", "gemv_coalesced", "gemv_fp8", "gemv_tc", "blocked_check", "gemv_checked", "gemv_tc_checked",
       "member_check", "sampling_check", "bank_build")  # fmt: skip
