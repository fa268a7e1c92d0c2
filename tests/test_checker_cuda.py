"""The trusted blocked checker on the GPU: its bank equals the reference's, its verdicts
equal the oracle's exact evaluation of the reference decision rule, and it meets the
reference's own GPU checker tests (tests/gpu/test_checker_cuda.py)."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import checker as ochk
from oracle.fp import U32, bf16, gamma, tree_height
from oracle.gemv import emulate_gemv
from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

GOLDEN = Path(__file__).parent / "golden"
M, N, THREADS = 512, 4100, 256
HEIGHT = tree_height(N, THREADS, vec=8)


def problem(m: int = M, n: int = N, seed: int = 0):
    W, x = inputs.numpy_problem(m, n, seed)
    return W, x, torch.from_numpy(W).to(torch.bfloat16).cuda(), torch.from_numpy(x).to(torch.bfloat16).cuda()


def make(Wt: torch.Tensor, block: int = 64, checks: int = 8, seed: int = 0, segments=None, height=HEIGHT):
    from pck.cuda import GpuBlockedChecker

    return GpuBlockedChecker(Wt, block, height, checks=checks, generator=torch.Generator().manual_seed(seed),
                             segments=segments)  # fmt: skip


def as_cuda(y: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32)).cuda()


def oracle_verdict(checker, x: np.ndarray, y: np.ndarray) -> dict:
    return ochk.gpu_verdict(checker.c.cpu().numpy(), checker.a.float().cpu().numpy(), checker.r.cpu().numpy(), x,
                            y, checker.coef, checker.geps, checker.tau_floor)  # fmt: skip


def assert_matches_oracle(checker, x: np.ndarray, y: np.ndarray, res) -> None:
    ref = oracle_verdict(checker, x, y)
    np.testing.assert_array_equal(res.passed.cpu().numpy(), ref["passed"])
    tau = res.tau.cpu().numpy()
    rho = res.rho.cpu().numpy()
    fin = np.isfinite(ref["tau"]) & np.isfinite(ref["rho"])
    assert np.all(tau[fin] >= ref["tau"][fin])  # never below the least sound threshold
    assert np.all(tau[fin] <= ref["tau"][fin] * (1 + 1e-9))
    # rho is the exact residual up to the kernel's own binary64 rounding, far inside tau
    assert np.all(np.abs(rho[fin] - ref["rho"][fin]) <= 1e-6 * ref["tau"][fin])
    # no case sits within rounding distance of the decision boundary
    ratio = np.abs(ref["rho"][fin]) / ref["tau"][fin]
    assert not np.any(np.abs(ratio - 1) < 1e-6)


def test_bank_matches_reference_bitwise() -> None:
    g = np.load(GOLDEN / "bank_small.npz")
    W, _, Wt, _ = problem(256, 1000, seed=1)
    ch = make(Wt, 32, 4, seed=1, segments=3, height=23)
    np.testing.assert_array_equal(ch.r.cpu().numpy(), g["r"])
    np.testing.assert_array_equal(ch.c.cpu().numpy().view(np.uint32), g["c"].view(np.uint32))
    np.testing.assert_array_equal(ch.a.view(torch.int16).cpu().numpy(), g["a"])
    assert [ch.coef, ch.geps, ch.tau_floor, ch.segments] == list(g["consts"])


def test_config1_bank_matches_reference() -> None:
    from pck.cuda import GpuBlockedChecker

    g = np.load(GOLDEN / "config1.npz")
    gen = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 4096, generator=gen) * 0.02).bfloat16()
    torch.randn(4096, generator=gen)  # x
    ch = GpuBlockedChecker(W.cuda(), 128, tree_height(4096, 256, 8), checks=1, generator=gen, segments=8)
    np.testing.assert_array_equal(ch.r.cpu().numpy(), g["r"])
    assert inputs.digest(ch.c.cpu().numpy()) == str(g["c_digest"])
    assert inputs.digest(ch.a.view(torch.int16).cpu().numpy()) == str(g["a_digest"])


@pytest.mark.parametrize("block", [1, 8, 64, 128, 512])
def test_legit_gpu_output_passes_and_matches_oracle(block: int) -> None:
    from pck.cuda import gemv_coalesced, gemv_naive

    _, x, Wt, xt = problem()
    checker = make(Wt, block)
    for y in (gemv_coalesced(Wt, xt, THREADS), gemv_naive(Wt, xt, THREADS)):
        res = checker.check(xt, y)
        assert res.passed.all()
        assert (res.rho.abs() <= res.tau).all()
    if block in (64, 512):
        assert_matches_oracle(checker, x, y.cpu().numpy(), res)


def test_matches_fp64_reference() -> None:
    """The reference's own tolerance test (tests/gpu/test_checker_cuda.py:54-80)."""
    from pck.cuda import GpuBlockedChecker, gemv_coalesced

    _, x, Wt, xt = problem(m=256, n=1000, seed=1)
    checker = GpuBlockedChecker(Wt, 32, HEIGHT, checks=4, generator=torch.Generator().manual_seed(1))
    y = gemv_coalesced(Wt, xt, 128)
    res = checker.check(xt, y)
    c = checker.c.cpu().numpy().astype(np.float64)
    a = checker.a.float().cpu().numpy().astype(np.float64)
    r = checker.r.cpu().numpy().astype(np.float64)
    x64, yb = x.astype(np.float64), y.cpu().numpy().astype(np.float64).reshape(-1, 32)
    rho = c @ x64 - np.einsum("kbi,bi->kb", r, yb)
    s = a @ np.abs(x64)
    bound = checker.geps * ((1 + U32) * s + np.abs(yb).sum(1)) + checker.tau_floor
    tau = (gamma(HEIGHT) + U32) * s + bound
    assert np.all(np.abs(res.rho.cpu().numpy() - rho) <= 2 * bound)
    tau_gpu = res.tau.cpu().numpy()
    assert np.all(tau_gpu >= tau * (1 - 1e-12))
    assert np.all(tau_gpu <= tau * (1 + 1e-3))
    assert_matches_oracle(checker, x, y.cpu().numpy(), res)


@pytest.mark.parametrize("exploit", ["skip_tail", "acc_bf16", "partial_bf16", "bf16_output"])
def test_planted_exploits_caught(exploit: str) -> None:
    from pck.cuda import GpuBlockedChecker

    W, x, Wt, xt = problem(m=512, n=2048, seed=2)
    checker = GpuBlockedChecker(Wt, 64, tree_height(2048, 128), checks=8, generator=torch.Generator().manual_seed(2))
    legit = emulate_gemv(W, x, 128)
    y = {
        "skip_tail": lambda: emulate_gemv(W, x, 128, drop_tail=4),
        "acc_bf16": lambda: emulate_gemv(W, x, 128, acc_bf16=True),
        "partial_bf16": lambda: emulate_gemv(W, x, 128, partial_bf16=True),
        "bf16_output": lambda: bf16(legit),
    }[exploit]()
    assert checker.verdict(xt, as_cuda(legit)).all()
    res = checker.check(xt, as_cuda(y))
    assert not res.verdict.all()
    assert_matches_oracle(checker, x, y, res)


@pytest.mark.parametrize("bad", [math.nan, math.inf, -math.inf])
def test_non_finite_output_fails_its_block_only(bad: float) -> None:
    from pck.cuda import gemv_coalesced

    _, _, Wt, xt = problem()
    checker = make(Wt, 64, checks=2)
    y = gemv_coalesced(Wt, xt, THREADS)
    y[130] = bad
    expected = np.ones(M // 64, dtype=bool)
    expected[130 // 64] = False
    np.testing.assert_array_equal(checker.verdict(xt, y).cpu().numpy(), expected)


def test_large_single_error_always_caught() -> None:
    from pck.cuda import gemv_coalesced

    _, _, Wt, xt = problem(seed=4)
    checker = make(Wt, 64, checks=8, seed=4)
    y = gemv_coalesced(Wt, xt, THREADS)
    tau = checker.check(xt, y).tau.min(dim=0).values
    for i in (torch.arange(0, M, 64 + 3) % M).tolist():
        bad = y.clone()
        bad[i] += 2.5 * float(tau[i // 64])
        verdict = checker.verdict(xt, bad)
        assert not verdict[i // 64]
        assert verdict.sum() == M // 64 - 1


def test_no_false_alarms_over_many_draws() -> None:
    from pck.cuda import gemv_coalesced

    _, _, Wt, xt = problem(seed=5)
    y = gemv_coalesced(Wt, xt, THREADS)
    for seed in range(50):
        assert make(Wt, 64, checks=8, seed=seed).verdict(xt, y).all()


@pytest.mark.parametrize(("kwargs", "match"), [({"block": 7}, "divide"), ({"block": 0}, "positive"),
                                                ({"block": 64, "checks": 0}, "checks")])  # fmt: skip
def test_rejects_bad_configuration(kwargs: dict, match: str) -> None:
    from pck.cuda import GpuBlockedChecker

    _, _, Wt, _ = problem(m=64, n=16)
    with pytest.raises(ValueError, match=match):
        GpuBlockedChecker(Wt, height=4, **kwargs)


def test_rejects_non_bf16_weights() -> None:
    from pck.cuda import GpuBlockedChecker

    with pytest.raises(ValueError, match="bfloat16"):
        GpuBlockedChecker(torch.ones((8, 8), device="cuda"), 4, 4)


@pytest.mark.parametrize(("which", "match"), [("y_dtype", "y must be"), ("y_shape", "shape"),
                                              ("x_dtype", "x must be"), ("y_cpu", "CUDA")])  # fmt: skip
def test_rejects_bad_check_inputs(which: str, match: str) -> None:
    from pck.cuda import GpuBlockedChecker

    _, _, Wt, xt = problem(m=64, n=16)
    checker = GpuBlockedChecker(Wt, 16, 4)
    y = torch.zeros(64, device="cuda")
    args = {"y_dtype": (xt, y.double()), "y_shape": (xt, y[:32]), "x_dtype": (xt.float(), y),
            "y_cpu": (xt, y.cpu())}[which]  # fmt: skip
    with pytest.raises(RuntimeError, match=match):
        checker.check(*args)


@pytest.mark.parametrize("segments", [1, 2, 3, 7, 64, 1000])
def test_segment_count_does_not_change_result(segments: int) -> None:
    from pck.cuda import gemv_coalesced

    _, x, Wt, xt = problem(m=256, n=1000, seed=6)
    y = gemv_coalesced(Wt, xt, 128)
    ref = make(Wt, 32, 4, seed=6, segments=1).check(xt, y)
    split_checker = make(Wt, 32, 4, seed=6, segments=segments)
    split = split_checker.check(xt, y)
    assert torch.equal(split.passed, ref.passed)
    assert bool(((split.rho - ref.rho).abs() <= 1e-4 * ref.tau).all())
    torch.testing.assert_close(split.tau, ref.tau, rtol=(1000 + 1) * 2.0**-24, atol=0)
    a = split_checker.a.float().cpu().numpy().astype(np.float64)
    s_exact = a @ np.abs(x.astype(np.float64))
    assert np.all(split.tau.cpu().numpy() >= (gamma(HEIGHT) + U32) * s_exact * (1 - 1e-12))


def test_repeated_calls_reuse_scratch_correctly() -> None:
    from pck.cuda import gemv_coalesced

    _, _, Wt, xt = problem(seed=7)
    checker = make(Wt, 64, checks=2)
    y = gemv_coalesced(Wt, xt, THREADS)
    bad = y.clone()
    bad[5] = math.nan
    first = checker.check(xt, y)
    for _ in range(20):
        assert torch.equal(checker.verdict(xt, bad)[1:], first.verdict[1:])
        assert not checker.verdict(xt, bad)[0]
        again = checker.check(xt, y)
        assert torch.equal(again.passed, first.passed)
        assert torch.equal(again.rho, first.rho)


@pytest.mark.parametrize("segments", [0, 1001])
def test_rejects_bad_segment_count(segments: int) -> None:
    from pck.cuda import GpuBlockedChecker

    _, _, Wt, _ = problem(m=64, n=1000)
    with pytest.raises(ValueError, match="segments"):
        GpuBlockedChecker(Wt, 16, 4, segments=segments)


def test_a_is_bf16_rounded_up_from_exact() -> None:
    from pck.cuda import GpuBlockedChecker

    W, _, Wt, _ = problem(m=256, n=1000, seed=8)
    checker = GpuBlockedChecker(Wt, 32, HEIGHT)
    a = checker.a.float().cpu().numpy().astype(np.float64)
    exact = np.abs(W.astype(np.float64)).reshape(256 // 32, 32, 1000).sum(axis=1)
    assert checker.a.dtype == torch.bfloat16
    assert np.all(a >= exact) and np.all(a <= exact * (1 + 2.0**-7))


@pytest.mark.parametrize("scale_exp", [-100, -120, 60])
def test_legit_output_passes_at_extreme_scales(scale_exp: int) -> None:
    from pck.cuda import GpuBlockedChecker, gemv_coalesced

    rng = np.random.default_rng(9)
    W = inputs.bf16_round(rng.standard_normal((256, 2048)) * 0.02)
    x = inputs.bf16_round(rng.standard_normal(2048) * 2.0**scale_exp)
    Wt, xt = torch.from_numpy(W).to(torch.bfloat16).cuda(), torch.from_numpy(x).to(torch.bfloat16).cuda()
    checker = GpuBlockedChecker(Wt, 64, tree_height(2048, 128, vec=8), checks=8,
                                generator=torch.Generator().manual_seed(9))  # fmt: skip
    y = gemv_coalesced(Wt, xt, 128)
    assert torch.isfinite(y).all()
    res = checker.check(xt, y)
    assert res.verdict.all()
    assert_matches_oracle(checker, x, y.cpu().numpy(), res)


def test_an_overflowing_threshold_fails_closed() -> None:
    m, n = 128, 4096
    signs = torch.where(torch.arange(n) % 2 == 0, 1.0, -1.0)
    Wt = (signs * 2.0**100).repeat(m, 1).to(torch.bfloat16).cuda()
    xt = torch.full((n,), 2.0**24).to(torch.bfloat16).cuda()
    checker = make(Wt, 64, checks=2)
    res = checker.check(xt, torch.full((m,), 1e30, device="cuda"))
    assert not torch.isfinite(res.tau).any()
    assert not res.passed.any()


@pytest.mark.parametrize("settled", [False, True])
def test_bank_built_just_before_a_checked_launch(settled: bool) -> None:
    """pck_bank_build directly followed, on the same stream and with no synchronization, by a
    checked launch that reads the new bank: the launch waits for the bank kernel before it
    reads c and a (the bank CTAs prefetch only for checks flagged PCK_CHECK_BANK_SETTLED, which
    this one is not), so the verdicts equal those of the same launch run after a synchronize.
    Settled weights (PCK_WEIGHTS_SETTLED) change nothing here: only W, written long before, is
    read early."""
    import ctypes

    from pck.cuda import _lib
    from pck.cuda._ext import extension, stream_handle
    from pck.fp import sum_up_factor

    W, x, Wt, xt = problem(1024, 4096, seed=5)
    ch = make(Wt, block=128, checks=2, seed=9, height=tree_height(4096, THREADS, 8))
    lib = _lib.library()
    ext = extension()
    stream = stream_handle(Wt.device)

    def launch(c, a):
        y = torch.empty(1024, dtype=torch.float32, device="cuda")
        desc = _lib.CheckDesc()
        _, _, r, pcx, ps, ctr, coef, geps, floor = ch.check_args(xt)
        out = ext.describe(c, a, r, xt, y, pcx, ps, ctr, coef, geps, floor, Wt.device, desc)
        job = (_lib.GemvJob * 1)()
        job[0].W, job[0].X, job[0].Y = Wt.data_ptr(), xt.data_ptr(), y.data_ptr()
        job[0].m, job[0].n, job[0].batch, job[0].threads = 1024, 4096, 1, THREADS
        job[0].weight_format = _lib.PCK_WEIGHTS_BF16 | (_lib.PCK_WEIGHTS_SETTLED if settled else 0)
        job[0].check = ctypes.pointer(desc)
        _lib.check(lib.pck_gemv_checked(job, 1, stream))
        return y, out

    torch.cuda.synchronize()
    for trial in range(3):
        c = torch.full_like(ch.c, float("nan"))  # a stale bank would fail every block
        a = torch.full_like(ch.a, float("nan"))
        torch.cuda.synchronize()
        _lib.check(lib.pck_bank_build(Wt.data_ptr(), ch.r.data_ptr(), c.data_ptr(), a.data_ptr(), 1024, 4096,
                                      128, 2, float(sum_up_factor(128)), stream))  # fmt: skip
        y, (passed, rho, tau) = launch(c, a)
        torch.cuda.synchronize()
        assert bool(passed.all()), f"trial {trial}: a block failed against a bank built just before"
        y0, (passed0, rho0, tau0) = launch(ch.c, ch.a)
        torch.cuda.synchronize()
        assert torch.equal(y, y0) and torch.equal(passed, passed0)
        assert torch.equal(rho, rho0) and torch.equal(tau, tau0)
