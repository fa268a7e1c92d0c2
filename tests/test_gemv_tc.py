"""The tensor-core batched GEMV (tcgen05): every output within the declared accumulation bound
of the exact product, the blocked checker built with `tc_height` raises no false alarm on
its outputs and catches planted faults."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

U32 = 2.0**-24


def problem(m: int, n: int, batch: int, seed: int):
    W, _ = inputs.torch_problem(m, n, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1)
    X = torch.randn(batch, n, generator=gen)
    X[:, torch.randperm(n, generator=gen)[: max(1, n // 100)]] *= 20.0  # outlier channels
    return W.cuda(), X.bfloat16().cuda()


def bound_ratio(W: torch.Tensor, X: torch.Tensor, Y: torch.Tensor) -> float:
    """max |Y - exact| / (gamma_h(u32) sum |w||x|) over all outputs (<= 1 within the bound)."""
    from pck.cuda import tc_height
    from pck.fp import gamma

    W64, X64 = W.double(), X.double()
    exact = X64 @ W64.T
    mag = X64.abs() @ W64.abs().T
    err = (Y.double() - exact).abs()
    g = gamma(tc_height(W.size(1)), U32)
    ratio = err / (g * mag).clamp(min=1e-300)
    return float(ratio.max())


def assert_tau_matches(fused: torch.Tensor, standalone: torch.Tensor, n: int) -> None:
    """tau of a check reduced inside the tensor-core kernel against the standalone check's
    (binary64 bank sums): the kernel sums the bound row a . |x| in binary32 rounded up, never
    below the exact sum and above it by at most a relative (1 + 2^-23)^h - 1 for chains of
    h <= n additions, so tau is never smaller and larger by at most about n * 2^-23."""
    assert bool((fused >= standalone * (1 - 1e-12)).all())
    assert bool((fused <= standalone * (1 + 1.01 * n * 2.0**-23) + 1e-300).all())

@pytest.mark.parametrize(("m", "n", "batch"), [(128, 64, 16), (128, 4096, 64), (300, 1000, 50), (1024, 4096, 128),
                                               (512, 4096, 256), (128, 14336, 16), (640, 2048, 1)])  # fmt: skip
def test_outputs_within_the_declared_bound(m: int, n: int, batch: int) -> None:
    from pck.cuda import gemv_tc

    W, X = problem(m, n, batch, seed=m + n + batch)
    Y = gemv_tc(W, X)
    assert Y.shape == (batch, m) and torch.isfinite(Y).all()
    ratio = bound_ratio(W, X, Y)
    print(f"tc bound ratio m={m} n={n} batch={batch}: {ratio:.3e}")
    assert ratio <= 1.0
    # and close to the product in plain terms
    ref = (X.double() @ W.double().T).float()
    torch.testing.assert_close(Y, ref, rtol=1e-3, atol=1e-3)


def test_decode_layer_shapes_and_repeat_calls() -> None:
    from pck.cuda import gemv_tc

    for m, n in [(6144, 4096), (4096, 14336)]:
        W, X = problem(m, n, 128, seed=m)
        Y1 = gemv_tc(W, X)
        Y2 = gemv_tc(W, X)
        assert torch.equal(Y1, Y2)  # deterministic
        assert bound_ratio(W, X, Y1) <= 1.0


def test_checker_with_tc_height_no_false_alarm_and_catches_faults() -> None:
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    m, n, batch = 1024, 4096, 128
    W, X = problem(m, n, batch, seed=5)
    Y = gemv_tc(W, X)
    checker = GpuBlockedChecker(W, 128, tc_height(n), checks=2, generator=torch.Generator().manual_seed(0))
    for b0 in range(0, batch, 16):
        res = checker.check(X[b0 : b0 + 16].contiguous(), Y[b0 : b0 + 16].contiguous())
        assert res.verdict.all()
        assert float((res.rho.abs() / res.tau).max()) < 1.0
    honest = checker.check(X[96:112].contiguous(), Y[96:112].contiguous())
    bad = Y.clone()
    bad.view(torch.int32)[7, 300] ^= 1 << 30  # exponent flip
    bad[100, 777] += 4.0 * float(honest.tau[4, :, 777 // 128].max())  # 4 tau: above the 2 tau guarantee
    res = checker.check(X[0:16].contiguous(), bad[0:16].contiguous())
    assert not res.verdict[7, 300 // 128]
    res = checker.check(X[96:112].contiguous(), bad[96:112].contiguous())
    assert not res.verdict[4, 777 // 128]


def test_rejects_unsupported_inputs() -> None:
    from pck.cuda import gemv_tc

    W, X = problem(128, 64, 16, seed=1)
    with pytest.raises(RuntimeError, match="bfloat16"):
        gemv_tc(W.float(), X)
    with pytest.raises(RuntimeError, match="batch"):
        gemv_tc(W, torch.zeros(257, 64, dtype=torch.bfloat16, device="cuda"))
    W2, X2 = problem(128, 60, 16, seed=2)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        gemv_tc(W2, X2)
    assert gemv_tc(W[:0], X).shape == (16, 0)


def test_tc_height_is_conservative_in_the_chain_length() -> None:
    from pck.cuda import tc_height

    assert tc_height(16) == 16 and tc_height(4096) == 8 * 257 and tc_height(4097) == 8 * 258
    assert np.all(np.diff([tc_height(n) for n in range(1, 2000)]) >= 0)


@pytest.mark.parametrize(("m", "n", "batch", "checks"), [(1024, 4096, 128, 1), (384, 1000, 50, 3), (512, 4096, 256, 8),
                                                         (256, 14336, 16, 2)])  # fmt: skip
def test_checked_call_matches_the_standalone_check(m: int, n: int, batch: int, checks: int) -> None:
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    W, X = problem(m, n, batch, seed=m * 3 + batch)
    checker = GpuBlockedChecker(W, 128, tc_height(n), checks=checks, generator=torch.Generator().manual_seed(9))
    Y, res = gemv_tc(W, X, checker)
    assert torch.equal(Y.view(torch.int32), gemv_tc(W, X).view(torch.int32))  # the check leaves Y alone
    assert res.passed.shape == (batch, checks, m // 128) and res.verdict.all()
    for b0 in range(0, batch, 16):
        sep = checker.check(X[b0 : b0 + 16].contiguous(), Y[b0 : b0 + 16].contiguous())
        assert torch.equal(sep.passed, res.passed[b0 : b0 + 16])
        assert_tau_matches(res.tau[b0 : b0 + 16], sep.tau, n)
        assert float(((res.rho[b0 : b0 + 16] - sep.rho).abs() / sep.tau).max()) < 1e-6


def test_checked_call_catches_a_bank_for_other_weights() -> None:
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    W, X = problem(512, 4096, 64, seed=77)
    W2 = W.clone()
    W2[5::128] += 1.0  # one row of every block changed: |delta y| ~ 100, far above 2 tau
    checker = GpuBlockedChecker(W2, 128, tc_height(4096), checks=2, generator=torch.Generator().manual_seed(1))
    _, res = gemv_tc(W, X, checker)
    delta = (X.double() @ (W2.double() - W.double()).T).abs().view(64, 4, 128).amax(dim=2)
    assert bool((delta > 2 * res.tau.amax(dim=1)).all())
    assert not res.verdict.any()


def e4m3_problem(m: int, n: int, batch: int, seed: int):
    from pck.cuda import quantize_fp8

    W, X = problem(m, n, batch, seed)
    Q, _ = quantize_fp8(W)
    return Q, X


@pytest.mark.parametrize(("m", "n", "batch"), [(128, 64, 16), (1024, 4096, 128), (384, 4096, 64), (300, 1008, 50), (19200, 4096, 64),
                                               (512, 4096, 256), (256, 14336, 16)])  # fmt: skip
def test_e4m3_weights_within_the_declared_bound(m: int, n: int, batch: int) -> None:
    """E4M3 weights on the tensor cores: widened exactly to bfloat16 in shared memory, so the
    outputs are those of the bfloat16 path on Q widened, within the same declared bound."""
    from pck.cuda import gemv_tc

    Q, X = e4m3_problem(m, n, batch, seed=m + n)
    Y = gemv_tc(Q, X)
    Qb = Q.to(torch.bfloat16)
    assert bound_ratio(Qb, X, Y) <= 1.0
    assert torch.equal(Y.view(torch.int32), gemv_tc(Qb, X).view(torch.int32))


@pytest.mark.parametrize(("m", "n", "batch", "checks", "fmt"),
                         [(1024, 4096, 128, 1, "bf16"), (384, 1000, 50, 3, "bf16"), (4096, 4096, 64, 4, "bf16"),
                          (512, 4096, 256, 2, "bf16"), (37888, 4096, 64, 1, "bf16"), (1024, 4096, 128, 2, "e4m3"),
                          (640, 14336, 32, 1, "e4m3"), (2048, 4096, 8, 1, "bf16")])  # fmt: skip
def test_fused_bank_sums_match_the_standalone_check(m: int, n: int, batch: int, checks: int, fmt: str) -> None:
    """The checks whose bank rows the tensor-core kernel reduces itself (persistent units of
    two tiles and split-K clusters, every batch width) decide exactly as the standalone check
    on the same outputs: every block passes, the bits are equal, tau agrees within the
    binary32 rounding of the bound row and rho is far inside tau."""
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    if fmt == "e4m3":
        W, X = e4m3_problem(m, n, batch, seed=m + checks)
        Wb = W.to(torch.bfloat16)
    else:
        W, X = problem(m, n, batch, seed=m + checks)
        Wb = W
    checker = GpuBlockedChecker(Wb, 128, tc_height(n), checks=checks, generator=torch.Generator().manual_seed(4))
    Y, res = gemv_tc(W, X, checker)
    assert torch.equal(Y.view(torch.int32), gemv_tc(W, X).view(torch.int32))
    assert res.verdict.all()
    for b0 in range(0, batch, 16):
        b1 = min(batch, b0 + 16)
        sep = checker.check(X[b0:b1].contiguous(), Y[b0:b1].contiguous())
        assert torch.equal(sep.passed, res.passed[b0:b1])
        assert_tau_matches(res.tau[b0:b1], sep.tau, n)
        assert float(((res.rho[b0:b1] - sep.rho).abs() / sep.tau).max()) < 1e-6


def test_fused_check_catches_planted_weights() -> None:
    """A bank built for other weights: the fused reduction fails every block whose output
    moved by more than 2 tau (the guaranteed case), at every batch width."""
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    W, X = problem(1024, 4096, 128, seed=78)
    W2 = W.clone()
    W2[9::128] += 1.0  # one row of every block: |delta y| = |sum of x|
    checker = GpuBlockedChecker(W2, 128, tc_height(4096), checks=1, generator=torch.Generator().manual_seed(2))
    _, res = gemv_tc(W, X, checker)
    delta = (X.double() @ (W2.double() - W.double()).T).abs().view(128, 8, 128).amax(dim=2)
    guaranteed = delta > 2 * res.tau.amax(dim=1)
    assert int(guaranteed.sum()) > 900
    assert not bool(res.verdict[guaranteed].any())
    from pck.cuda import device_status

    assert device_status() == 0


def test_fused_bank_sums_with_zeros_and_subnormal_activations() -> None:
    """Activations with exact zeros (both signs), bfloat16 subnormals and large values take
    every branch of the bank warps' widening to binary64; the fused sums still decide as the
    standalone check does."""
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height

    W, X = problem(2048, 4096, 64, seed=91)
    gen = torch.Generator().manual_seed(92)
    Xc = X.cpu().float()
    pick = torch.rand(Xc.shape, generator=gen)
    Xc[pick < 0.10] = 0.0
    Xc[(pick >= 0.10) & (pick < 0.12)] = -0.0
    Xc[(pick >= 0.12) & (pick < 0.14)] = 3e-39  # subnormal in bfloat16
    Xc[(pick >= 0.14) & (pick < 0.15)] = -1e30
    X = Xc.bfloat16().cuda()
    checker = GpuBlockedChecker(W, 128, tc_height(4096), checks=2, generator=torch.Generator().manual_seed(6))
    Y, res = gemv_tc(W, X, checker)
    for b0 in range(0, 64, 16):
        sep = checker.check(X[b0 : b0 + 16].contiguous(), Y[b0 : b0 + 16].contiguous())
        assert torch.equal(sep.passed, res.passed[b0 : b0 + 16])
        assert_tau_matches(res.tau[b0 : b0 + 16], sep.tau, 4096)
