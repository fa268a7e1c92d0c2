"""Batched checks and the fused checked GEMV (the reference's tests/gpu/test_check_many.py
and tests/gpu/test_side_stream.py, plus the one-launch GEMV + check of this build)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import checker as ochk
from oracle.fp import tree_height

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

THREADS = 128
CONFIGS = [  # (m, n, block, checks, segments)
    (512, 4096, 64, 1, None),
    (1024, 512, 32, 2, 1),
    (256, 14336, 128, 4, 7),
    (64, 1000, 8, 1, 3),
    (2048, 4096, 256, 2, None),
]


def make(m: int, n: int, block: int, checks: int, segments, seed: int):
    from pck.cuda import GpuBlockedChecker, gemv_coalesced

    gen = torch.Generator().manual_seed(seed)
    W = (torch.randn(m, n, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    x = torch.randn(n, generator=gen).to(torch.bfloat16).cuda()
    checker = GpuBlockedChecker(W, block, tree_height(n, THREADS, vec=8), checks=checks, generator=gen,
                                segments=segments)  # fmt: skip
    return checker, x, gemv_coalesced(W, x, THREADS), W


def test_batch_matches_individual_checks() -> None:
    from pck.cuda import check_many

    items = [make(*cfg, seed=i) for i, cfg in enumerate(CONFIGS)]
    batched = check_many([it[:3] for it in items])
    for (checker, x, y, _), res in zip(items, batched, strict=True):
        alone = checker.check(x, y)
        assert torch.equal(res.passed, alone.passed)
        assert torch.equal(res.rho, alone.rho)
        assert torch.equal(res.tau, alone.tau)
        assert res.verdict.all()


def test_more_than_one_launch_and_fault_isolation() -> None:
    from pck.cuda import check_many

    items = [make(*CONFIGS[i % len(CONFIGS)], seed=10 + i)[:3] for i in range(11)]
    checker, x, y = items[9]
    bad = y.clone()
    bad[3] = float("inf")
    items[9] = (checker, x, bad)
    results = check_many(items)
    assert len(results) == 11
    for i, res in enumerate(results):
        if i == 9:
            assert not res.verdict[0] and res.verdict[1:].all()
        else:
            assert res.verdict.all()


def test_rejects_same_checker_twice() -> None:
    from pck.cuda import check_many

    item = make(*CONFIGS[0], seed=0)[:3]
    with pytest.raises(ValueError, match="once"):
        check_many([item, item])


def test_extension_rejects_bad_batches() -> None:
    from pck.cuda._ext import extension

    checker, x, y, _ = make(*CONFIGS[0], seed=0)
    args = [checker.c, checker.a, checker.r, x, y, checker._partial_cx, checker._partial_s, checker._counters,
            checker.coef, checker.geps, checker.tau_floor]  # fmt: skip
    with pytest.raises(RuntimeError, match="batch size"):
        extension().blocked_check(*([] for _ in args))
    with pytest.raises(RuntimeError, match="batch size"):
        extension().blocked_check(*([a] * 9 for a in args))
    lists = [[a] for a in args]
    lists[4] = [y, y]
    with pytest.raises(RuntimeError, match="same length"):
        extension().blocked_check(*lists)


@pytest.mark.parametrize("cfg", CONFIGS)
def test_fused_gemv_and_check_equal_the_separate_launches(cfg) -> None:
    from pck.cuda import gemv_checked

    checker, x, y_sep, W = make(*cfg, seed=3)
    alone = checker.check(x, y_sep)
    y, res = gemv_checked(W, x, checker, THREADS)
    assert torch.equal(y.view(torch.int32), y_sep.view(torch.int32))  # same bits
    assert torch.equal(res.passed, alone.passed)
    assert torch.equal(res.rho, alone.rho)
    assert torch.equal(res.tau, alone.tau)
    assert res.verdict.all()


def test_layer_in_one_launch_matches_oracle() -> None:
    """q, k, v, o, gate, up, down of a Llama-3-8B layer (row counts scaled down 8x), each
    checked at b = 128, in one persistent launch."""
    from pck.cuda import GpuBlockedChecker, checked_gemvs

    shapes = [(512, 4096), (128, 4096), (128, 4096), (512, 4096), (1792, 4096), (1792, 4096), (512, 14336)]
    gen = torch.Generator().manual_seed(11)
    items = []
    for m, n in shapes:
        W = (torch.randn(m, n, generator=gen) * 0.02).bfloat16().cuda()
        x = torch.randn(n, generator=gen).bfloat16().cuda()
        items.append((W, x, GpuBlockedChecker(W, 128, tree_height(n, 256, 8), checks=1, generator=gen)))
    out = checked_gemvs(items, 256)
    from oracle.gemv import gemv_coalesced_c

    for (W, x, ch), (y, res) in zip(items, out, strict=True):
        ref_y = gemv_coalesced_c(W.view(torch.uint16).cpu().numpy(), x.view(torch.uint16).cpu().numpy(), 256, 8)
        np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), ref_y.view(np.uint32))
        ref = ochk.gpu_verdict(ch.c.cpu().numpy(), ch.a.float().cpu().numpy(), ch.r.cpu().numpy(),
                               x.float().cpu().numpy(), ref_y, ch.coef, ch.geps, ch.tau_floor)  # fmt: skip
        np.testing.assert_array_equal(res.passed.cpu().numpy(), ref["passed"])
        assert res.verdict.all()


def test_fused_check_catches_a_fault_planted_in_the_bank_path() -> None:
    """A fused launch whose y disagrees with the bank (the bank built for other weights)
    fails every block: the verdict reads y as stored and recomputes c . x independently."""
    from pck.cuda import GpuBlockedChecker, gemv_checked

    gen = torch.Generator().manual_seed(5)
    W = (torch.randn(512, 4096, generator=gen) * 0.02).bfloat16().cuda()
    W2 = W.clone()
    W2[::3] *= 1.5  # every block has perturbed rows
    x = torch.randn(4096, generator=gen).bfloat16().cuda()
    checker = GpuBlockedChecker(W2, 128, tree_height(4096, 256, 8), checks=2, generator=gen)
    _, res = gemv_checked(W, x, checker)
    assert not res.verdict.any()


def test_batched_check_columns_match_single_checks() -> None:
    from pck.cuda import GpuBlockedChecker, gemv_coalesced

    gen = torch.Generator().manual_seed(21)
    W = (torch.randn(1024, 4096, generator=gen) * 0.02).bfloat16().cuda()
    X = torch.randn(4, 4096, generator=gen).bfloat16().cuda()
    ch = GpuBlockedChecker(W, 128, tree_height(4096, 256, 8), checks=2, generator=gen)
    Y = gemv_coalesced(W, X, 256)
    Y[2, 300] += 1.0
    res = ch.check(X, Y)
    assert res.passed.shape == (4, 2, 8)
    for b in range(4):
        alone = ch.check(X[b].contiguous(), Y[b].contiguous())
        assert torch.equal(res.passed[b], alone.passed)
        assert torch.equal(res.rho[b], alone.rho)
    assert not res.verdict[2, 300 // 128] and res.verdict.sum() == 4 * 8 - 1


def test_side_stream_matches_same_stream() -> None:
    from pck.cuda import SideStreamChecker

    checker, x, y, _ = make(512, 4096, 64, 2, None, seed=0)
    serial = checker.check(x, y)
    result = SideStreamChecker().submit(checker, x, y).wait()
    assert torch.equal(result.passed, serial.passed)
    assert torch.equal(result.rho, serial.rho)
    assert torch.equal(result.tau, serial.tau)


def test_side_stream_sees_output_even_if_freed_and_overwritten() -> None:
    from pck.cuda import SideStreamChecker, gemv_coalesced

    checker, x, _, W = make(1024, 4096, 64, 2, None, seed=1)
    side = SideStreamChecker()
    pending = []
    for _ in range(20):
        y = gemv_coalesced(W, x, THREADS)
        pending.append(side.submit(checker, x, y))
        del y
        garbage = torch.full((1024,), float("nan"), device="cuda")
        garbage.add_(1)
    for p in pending:
        assert p.wait().verdict.all()


def test_one_verdict_launch_per_layer_equals_the_fused_launches() -> None:
    """GEMVs with deferred verdicts (pck_gemv_partials) and one verdict launch for every
    check of a scaled Llama-3-8B layer give the bits of the fused calls, including a block
    whose output was altered between the GEMV and the verdict."""
    from pck.cuda import GpuBlockedChecker
    from pck.cuda.plan import GemvLaunch, VerdictLaunch

    gen = torch.Generator().manual_seed(13)
    groups = [[(768, 4096), (128, 4096), (128, 4096)], [(512, 4096)], [(1792, 4096), (1792, 4096)],
              [(512, 14336)]]  # fmt: skip
    deferred, fused = [], []
    for shapes in groups:
        x = torch.randn(shapes[0][1], generator=gen).bfloat16().cuda()
        items = []
        for m, n in shapes:
            W = (torch.randn(m, n, generator=gen) * 0.02).bfloat16().cuda()
            items.append((W, x, GpuBlockedChecker(W, 128, tree_height(n, 256, 8), checks=2, generator=gen)))
        deferred.append(GemvLaunch(items, 256, verdicts=False))
        fused.append(GemvLaunch(items, 256))
    verdict = VerdictLaunch(deferred)
    for g in fused:
        g.launch()
    torch.cuda.synchronize()
    want = [[(y.clone(), r.passed.clone(), r.rho.clone(), r.tau.clone()) for y, r in zip(g.ys, g.results, strict=True)]
            for g in fused]  # fmt: skip
    for g in deferred:
        g.launch()
    deferred[1].ys[0][300] += 1.0  # a fault after the GEMV, before the verdicts
    verdict.launch()
    torch.cuda.synchronize()
    for gi, g in enumerate(deferred):
        for j, (y, r) in enumerate(zip(g.ys, g.results, strict=True)):
            y0, p0, rho0, tau0 = want[gi][j]
            if gi == 1:
                assert not bool(r.passed[:, 300 // 128].any()) and int(r.passed.sum()) == r.passed.numel() - 2
                continue
            assert torch.equal(y.view(torch.int32), y0.view(torch.int32))
            assert torch.equal(r.passed, p0) and torch.equal(r.rho, rho0) and torch.equal(r.tau, tau0)
            assert bool(r.passed.all())


def test_verdicts_carried_by_the_next_launch_equal_the_fused_launches() -> None:
    """pck_gemv_pipelined: every launch of a scaled Llama-3-8B layer decides the previous
    launch's checks (the first launch of the next layer decides the last), captured in a
    CUDA graph and replayed: the bits of the fused calls, and a fault planted between two
    launches is caught by the launch that decides it."""
    from pck.cuda import GpuBlockedChecker
    from pck.cuda.plan import GemvLaunch

    gen = torch.Generator().manual_seed(17)
    groups = [[(768, 4096), (128, 4096), (128, 4096)], [(512, 4096)], [(1792, 4096), (1792, 4096)],
              [(512, 14336)]]  # fmt: skip
    piped, fused = [], []
    for shapes in groups:
        x = torch.randn(shapes[0][1], generator=gen).bfloat16().cuda()
        items = []
        for m, n in shapes:
            W = (torch.randn(m, n, generator=gen) * 0.02).bfloat16().cuda()
            items.append((W, x, GpuBlockedChecker(W, 128, tree_height(n, 256, 8), checks=2, generator=gen)))
        piped.append(GemvLaunch(items, 256, verdicts=False))
        fused.append(GemvLaunch(items, 256))
    for i, g in enumerate(piped):
        g.set_prior([piped[i - 1]])  # the first launch decides the last one's checks
    for g in fused:
        g.launch()
    torch.cuda.synchronize()
    want = [[(y.clone(), r.passed.clone(), r.rho.clone(), r.tau.clone()) for y, r in zip(g.ys, g.results, strict=True)]
            for g in fused]  # fmt: skip

    def compare(skip_fault: bool) -> None:
        for gi, g in enumerate(piped):
            for j, (y, r) in enumerate(zip(g.ys, g.results, strict=True)):
                y0, p0, rho0, tau0 = want[gi][j]
                if skip_fault and gi == 1:
                    continue
                assert torch.equal(y.view(torch.int32), y0.view(torch.int32))
                assert torch.equal(r.passed, p0) and torch.equal(r.rho, rho0) and torch.equal(r.tau, tau0)
                assert bool(r.passed.all())

    # eager: a layer, then the next layer's first launch for the last verdicts
    for r in (res for g in piped for res in g.results):
        r.passed.zero_()
    for g in piped:
        g.launch()
    piped[0].launch()
    torch.cuda.synchronize()
    compare(False)

    # a fault between o's GEMV and the gate/up launch that decides o's blocks
    for g in piped[:2]:
        g.launch()
    piped[1].ys[0][300] += 1.0
    piped[2].launch()
    torch.cuda.synchronize()
    r = piped[1].results[0]
    assert not bool(r.passed[:, 300 // 128].any()) and int(r.passed.sum()) == r.passed.numel() - 2

    # graph: the cycle of four launches, replayed twice after a warm layer
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for g in piped:
            g.launch()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for g in piped:
                g.launch()
    torch.cuda.current_stream().wait_stream(stream)
    for _ in range(2):
        for r in (res for g in piped for res in g.results):
            r.passed.zero_()
        graph.replay()
        piped[0].launch()
        torch.cuda.synchronize()
        compare(False)
