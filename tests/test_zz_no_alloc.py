"""pck_gemv_checked_static, the checked GEMV whose check scratch is a fixed array inside the
library: through the C ABI it must give exactly what pck_gemv_checked gives on the same
inputs, call after call, and reject checks that need more scratch than the array holds.

Collected last on purpose: it must pass both alone in a fresh process (its first call then
does the per-device set-up) and after every other test has used the device."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.golden import inputs


def _lib():
    from pck.cuda import _lib

    return _lib


def checked_jobs(fmt: int, shapes: list[tuple[int, int, int]], seed: int):
    """(W, checker) per (m, n, checks), all with the same weight format."""
    from pck.cuda import GpuBlockedChecker, quantize_fp8
    from pck.fp import tree_height

    out = []
    for i, (m, n, checks) in enumerate(shapes):
        W, _ = inputs.torch_problem(m, n, seed=seed + i)
        W = W.cuda()
        vec = 8
        if fmt == _lib().PCK_WEIGHTS_E4M3:
            W = quantize_fp8(W)[0]
            vec = 16
        checker = GpuBlockedChecker(W.to(torch.bfloat16), 128, tree_height(n, 256, vec), checks=checks,
                                    generator=torch.Generator().manual_seed(seed + 100 + i))  # fmt: skip
        out.append((W, checker))
    return out


def activations(n: int, batch: int, seed: int) -> torch.Tensor:
    x = torch.stack([inputs.torch_problem(1, n, seed=seed + b)[1] for b in range(batch)])
    return (x if batch > 1 else x[0]).cuda()


def run_static(items, xs, fmt: int):
    """One pck_gemv_checked_static call: (y, passed, rho, tau) per job."""
    from pck.cuda._ext import extension, on_device, ptr, stream_handle

    lib = _lib()
    ext = extension()
    device = xs[0].device
    count = len(items)
    descs = (lib.CheckDesc * count)()
    arr = (lib.GemvJob * count)()
    results = []
    for g, ((W, checker), x) in enumerate(zip(items, xs, strict=True)):
        batch = x.size(0) if x.dim() == 2 else 1
        y = torch.full((*x.shape[:-1], W.size(0)), float("nan"), dtype=torch.float32, device=device)
        c, a, r, pcx, ps, ctr, coef, geps, floor = checker.check_args(x)
        passed, rho, tau = ext.describe(c, a, r, x, y, pcx, ps, ctr, coef, geps, floor, device, descs[g])
        descs[g].partial_cx = descs[g].partial_s = descs[g].counters = None  # the library's own
        job = arr[g]
        job.W, job.X, job.Y = ptr(W), ptr(x), ptr(y)
        job.m, job.n = W.size(0), W.size(1)
        job.batch, job.threads, job.weight_format = batch, 256, fmt
        job.check = ctypes.pointer(descs[g])
        results.append((y, passed, rho, tau))
    with on_device(device):
        rc = lib.library().pck_gemv_checked_static(arr, count, stream_handle(device))
    lib.check(rc, "pck_gemv_checked_static")
    return results


def run_existing(items, xs, fmt: int):
    """The same jobs through pck_gemv_checked, with each checker's own scratch."""
    from pck.cuda._ext import extension

    jobs = []
    ys = []
    for (W, checker), x in zip(items, xs, strict=True):
        y = torch.empty((*x.shape[:-1], W.size(0)), dtype=torch.float32, device=x.device)
        ys.append(y)
        jobs.append((W, x, y, checker.check_args(x)))
    outs = extension().gemv_checked(jobs, 256, fmt)
    return [(y, *out) for y, out in zip(ys, outs, strict=True)]


def assert_same(got, want) -> None:
    """Bit-identical y, verdicts, rho and tau (the kernel and its plan are the same)."""
    for (y, passed, rho, tau), (y0, passed0, rho0, tau0) in zip(got, want, strict=True):
        np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), y0.cpu().numpy().view(np.uint32))
        assert torch.equal(passed, passed0)
        np.testing.assert_array_equal(rho.cpu().numpy().view(np.uint64), rho0.cpu().numpy().view(np.uint64))
        np.testing.assert_array_equal(tau.cpu().numpy().view(np.uint64), tau0.cpu().numpy().view(np.uint64))
        assert bool(passed.all())


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
@pytest.mark.parametrize(
    ("fmt_name", "shapes", "batch"),
    [("bf16", [(1024, 4096, 2), (512, 2048, 1)], 1),
     ("bf16", [(768, 1024, 3)], 3),
     ("e4m3", [(1024, 4096, 2), (256, 4096, 1)], 2)],
)  # fmt: skip
def test_two_calls_in_a_row_match_the_allocating_entry_point(fmt_name: str, shapes, batch: int) -> None:
    lib = _lib()
    fmt = lib.PCK_WEIGHTS_BF16 if fmt_name == "bf16" else lib.PCK_WEIGHTS_E4M3
    items = checked_jobs(fmt, shapes, seed=11)
    first = [activations(n, batch, seed=500 + 7 * i) for i, (_, n, _) in enumerate(shapes)]
    second = [activations(n, batch, seed=900 + 7 * i) for i, (_, n, _) in enumerate(shapes)]
    got1 = run_static(items, first, fmt)
    got2 = run_static(items, second, fmt)
    torch.cuda.synchronize()
    want1 = run_existing(items, first, fmt)
    want2 = run_existing(items, second, fmt)
    torch.cuda.synchronize()
    assert_same(got1, want1)
    assert_same(got2, want2)
    assert lib.device_status() == 0


def test_rejects_checks_beyond_the_static_limit() -> None:
    """A check needing more than PCK_STATIC_SCRATCH_BYTES is refused before any device work,
    so this runs without a GPU."""
    lib = _lib()
    d = lib.CheckDesc()
    d.c = d.a = d.r = d.x = d.y = d.passed = d.rho = d.tau = 16
    d.n, d.block, d.num_blocks, d.checks, d.segments, d.batch = 4096, 128, 1024, 8, 64, 1
    d.coef = d.geps = d.tau_floor = 1.0
    need = 8 * 1 * (8 + 1) * 1024 * 64
    assert need > lib.STATIC_SCRATCH_BYTES
    job = (lib.GemvJob * 1)()
    job[0].W = job[0].X = job[0].Y = 16
    job[0].m, job[0].n, job[0].batch, job[0].threads = 1024 * 128, 4096, 1, 256
    job[0].check = ctypes.pointer(d)
    rc = lib.library().pck_gemv_checked_static(job, 1, None)
    assert rc == 1
    assert "static limit" in lib.library().pck_last_error().decode()


def test_rejects_jobs_that_fit_alone_but_not_together() -> None:
    """Two checks of 2.125 MiB of scratch each fit the array alone but not together: the call
    is refused with the summed size, before any device work (so no GPU is needed)."""
    lib = _lib()
    count = 2
    descs = (lib.CheckDesc * count)()
    jobs = (lib.GemvJob * count)()
    for g in range(count):
        d = descs[g]
        d.c = d.a = d.r = d.x = d.y = d.passed = d.rho = d.tau = 16 * (g + 1)
        d.n, d.block, d.num_blocks, d.checks, d.segments, d.batch = 4096, 128, 256, 16, 64, 1
        d.coef = d.geps = d.tau_floor = 1.0
        jobs[g].W = jobs[g].X = jobs[g].Y = 16 * (g + 1)
        jobs[g].m, jobs[g].n, jobs[g].batch, jobs[g].threads = 256 * 128, 4096, 1, 256
        jobs[g].check = ctypes.pointer(d)
    one = 8 * 16 * 256 * 64 + 8 * 256 * 64  # c . x partials, then a . |x| partials
    assert one <= lib.STATIC_SCRATCH_BYTES < count * one
    rc = lib.library().pck_gemv_checked_static(jobs, count, None)
    assert rc == 1  # PCK_ERR_ARGUMENT
    msg = lib.library().pck_last_error().decode()
    assert f"need {count * one} bytes" in msg and "static limit" in msg
