"""GPU GEMV kernels: bit-exact with the oracle and with the reference's golden outputs
(the reference's tests/gpu/test_gemv_cuda.py cases, plus batched columns)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle.gemv import emulate_gemv, emulate_gemv_coalesced, gemv_coalesced_c
from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

GOLDEN = np.load(Path(__file__).parent / "golden" / "gemv.npz")
CASES = [
    (1, 1, 32), (3, 5, 64), (7, 100, 32), (64, 1000, 32), (5, 17, 1024), (33, 4096, 128),
    (256, 4096, 256), (256, 4100, 256), (16, 14336, 512), (128, 4096, 1024), (9, 77, 64),
]  # fmt: skip


def cuda_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).cuda()


def bits(y: torch.Tensor) -> np.ndarray:
    return y.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize(("m", "n", "t"), CASES)
def test_coalesced_matches_reference_golden(m: int, n: int, t: int) -> None:
    from pck.cuda import gemv_coalesced

    W, x = inputs.numpy_problem(m, n, seed=m * n + t)
    np.testing.assert_array_equal(bits(gemv_coalesced(cuda_bf16(W), cuda_bf16(x), t)), GOLDEN[f"coalesced_{m}x{n}_t{t}"])


@pytest.mark.parametrize(("m", "n", "t"), CASES)
def test_naive_matches_reference_golden(m: int, n: int, t: int) -> None:
    from pck.cuda import gemv_naive

    W, x = inputs.numpy_problem(m, n, seed=m * n + t)
    np.testing.assert_array_equal(bits(gemv_naive(cuda_bf16(W), cuda_bf16(x), t)), GOLDEN[f"naive_{m}x{n}_t{t}"])


@pytest.mark.parametrize("threads", [1, 2, 4, 16, 32, 256])
def test_naive_small_thread_counts(threads: int) -> None:
    from pck.cuda import gemv_naive

    W, x = inputs.numpy_problem(9, 77, seed=threads)
    np.testing.assert_array_equal(bits(gemv_naive(cuda_bf16(W), cuda_bf16(x), threads)), GOLDEN[f"naive_small_t{threads}"])


@settings(max_examples=60, deadline=None)
@given(st.integers(1, 40), st.integers(1, 700), st.sampled_from([32, 64, 128, 256, 512, 1024]),
       st.integers(0, 2**32 - 1), st.sampled_from(["gauss", "student-t", "mixed-scale"]))  # fmt: skip
def test_coalesced_random_problems_match_oracle(m: int, n: int, t: int, seed: int, dist: str) -> None:
    from pck.cuda import gemv_coalesced, gemv_naive

    rng = np.random.default_rng(seed)
    W = inputs.bf16_round(rng.standard_normal((m, n)) * 0.02)
    if dist == "gauss":
        x = rng.standard_normal(n)
    elif dist == "student-t":
        x = rng.standard_t(3, n)
    else:
        x = rng.standard_normal(n) * 2.0 ** rng.integers(-20, 20, n)
    x = inputs.bf16_round(x)
    Wt, xt = cuda_bf16(W), cuda_bf16(x)
    np.testing.assert_array_equal(bits(gemv_coalesced(Wt, xt, t)), emulate_gemv_coalesced(W, x, t).view(np.uint32))
    np.testing.assert_array_equal(bits(gemv_naive(Wt, xt, t)), emulate_gemv(W, x, t).view(np.uint32))


@pytest.mark.parametrize(("m", "n"), [(4096, 4096), (1024, 14336), (14336, 4096)])
def test_full_size_shapes_match_c_oracle(m: int, n: int) -> None:
    """Decode-layer shapes through the staged (cp.async.bulk) path, against the C oracle."""
    from pck.cuda import gemv_coalesced

    W, x = inputs.torch_problem(m, n, seed=m + n)
    y = gemv_coalesced(W.cuda(), x.cuda(), 256)
    ref = gemv_coalesced_c(W.view(torch.uint16).numpy(), x.view(torch.uint16).numpy(), 256, 8)
    np.testing.assert_array_equal(bits(y), ref.view(np.uint32))


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8, 16])
@pytest.mark.parametrize("threads", [32, 256, 1024])
def test_batched_columns_each_match_the_single_tree(batch: int, threads: int) -> None:
    from pck.cuda import gemv_coalesced

    m, n = 200, 4096
    W, _ = inputs.torch_problem(m, n, seed=batch)
    X = (torch.randn(batch, n, generator=torch.Generator().manual_seed(batch)) * 2).bfloat16()
    Y = gemv_coalesced(W.cuda(), X.cuda(), threads)
    assert Y.shape == (batch, m)
    ref = gemv_coalesced_c(W.view(torch.uint16).numpy(), X.view(torch.uint16).numpy(), threads, 8)
    np.testing.assert_array_equal(bits(Y), ref.view(np.uint32))


def test_unaligned_pointer_uses_scalar_path() -> None:
    from pck.cuda import gemv_coalesced

    m, n, threads = 8, 4096, 128
    W, x = inputs.numpy_problem(m, n, seed=3)
    flat = torch.zeros(m * n + 1, dtype=torch.bfloat16, device="cuda")
    flat[1:] = cuda_bf16(W).flatten()
    view = flat[1:].view(m, n)
    assert view.is_contiguous() and view.data_ptr() % 16 != 0
    np.testing.assert_array_equal(bits(gemv_coalesced(view, cuda_bf16(x), threads)),
                                  emulate_gemv_coalesced(W, x, threads).view(np.uint32))  # fmt: skip


@pytest.mark.parametrize("kernel", ["naive", "coalesced"])
def test_signed_zero_matches_reference(kernel: str) -> None:
    from pck.cuda import gemv_coalesced, gemv_naive

    fn = gemv_naive if kernel == "naive" else gemv_coalesced
    W = torch.zeros((2, 64), dtype=torch.bfloat16, device="cuda")
    x = -torch.ones(64, dtype=torch.bfloat16, device="cuda")
    for t in (32, 64):
        np.testing.assert_array_equal(bits(fn(W, x, t)), GOLDEN[f"signed_zero_{kernel}_t{t}"])


@pytest.mark.parametrize("kernel", ["naive", "coalesced"])
def test_empty_output(kernel: str) -> None:
    from pck.cuda import gemv_coalesced, gemv_naive

    fn = gemv_naive if kernel == "naive" else gemv_coalesced
    W = torch.zeros((0, 8), dtype=torch.bfloat16, device="cuda")
    assert fn(W, torch.zeros(8, dtype=torch.bfloat16, device="cuda"), 32).shape == (0,)


@pytest.mark.parametrize("kernel", ["naive", "coalesced"])
@pytest.mark.parametrize(
    ("make", "match"),
    [
        (lambda W, x: (W.float(), x.float(), 32), "bfloat16"),
        (lambda W, x: (W.t(), x[:4], 32), "contiguous"),
        (lambda W, x: (W, x[:3], 32), "shape"),
        (lambda W, x: (W, x, 48), "power of two"),
        (lambda W, x: (W, x, 2048), "power of two"),
        (lambda W, x: (W.cpu(), x.cpu(), 32), "CUDA tensors"),
    ],
)
def test_rejects_bad_inputs(kernel: str, make, match: str) -> None:
    from pck.cuda import gemv_coalesced, gemv_naive

    fn = gemv_naive if kernel == "naive" else gemv_coalesced
    W = torch.ones((4, 8), dtype=torch.bfloat16, device="cuda")
    x = torch.ones(8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match=match):
        fn(*make(W, x))


def test_coalesced_rejects_fewer_than_a_warp() -> None:
    from pck.cuda import gemv_coalesced

    W = torch.ones((4, 8), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match=r"\[32, 1024\]"):
        gemv_coalesced(W, torch.ones(8, dtype=torch.bfloat16, device="cuda"), 16)


def test_no_bounded_wait_gave_up() -> None:
    from pck.cuda import device_status

    assert device_status(clear=True) == 0


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
@pytest.mark.parametrize("fmt", ["bf16", "e4m3"])
def test_chained_launches_with_next_prefetch_give_the_same_bits(fmt: str) -> None:
    """Launches chained with set_next (pck_gemv_pipelined_next: the CTAs prefetch the next
    launch's first weight pieces into L2) give the bits of the unchained calls, and the checks
    decided by the following launch pass."""
    from pck.cuda import GpuBlockedChecker, gemv_coalesced, gemv_fp8, quantize_fp8
    from pck.cuda.plan import GemvLaunch
    from pck.fp import tree_height

    gen = torch.Generator(device="cuda").manual_seed(21)
    shapes = [(3072, 4096), (1024, 4096), (2048, 14336)]
    launches, refs = [], []
    for i, (m, n) in enumerate(shapes):
        W = (torch.randn(m, n, generator=gen, device="cuda") * 0.02).bfloat16()
        x = torch.randn(n, generator=gen, device="cuda").bfloat16()
        vec = 8
        if fmt == "e4m3":
            W, vec = quantize_fp8(W)[0], 16
        ch = GpuBlockedChecker(W.to(torch.bfloat16), 128, tree_height(n, 256, vec),
                               generator=torch.Generator().manual_seed(i))  # fmt: skip
        launches.append(GemvLaunch([(W, x, ch)], 256, verdicts=False))
        refs.append(gemv_fp8(W, x) if fmt == "e4m3" else gemv_coalesced(W, x))
    for i, g in enumerate(launches):
        g.set_prior([launches[i - 1]])
        g.set_next(launches[(i + 1) % len(launches)])
    for _ in range(3):
        for g in launches:
            g.launch()
    launches[0].launch()  # decides the last launch's checks
    torch.cuda.synchronize()
    for g, ref in zip(launches, refs, strict=True):
        assert torch.equal(g.ys[0].view(torch.int32), ref.view(torch.int32))
        assert bool(g.results[0].passed.all())


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_settled_bank_gives_the_same_verdicts() -> None:
    """Checks flagged PCK_CHECK_BANK_SETTLED (GemvLaunch's default: the bank CTAs request
    their first pieces before the producer wait) decide every block as the same launches
    without the flag, rho and tau bit for bit, with one planted fault caught either way;
    unknown check flags are rejected."""
    from pck.cuda import GpuBlockedChecker, _lib
    from pck.cuda.plan import GemvLaunch
    from pck.fp import tree_height

    gen = torch.Generator(device="cuda").manual_seed(5)
    items = []
    for i, (m, n) in enumerate([(1024, 4096), (512, 14336)]):
        W = (torch.randn(m, n, generator=gen, device="cuda") * 0.02).bfloat16()
        x = torch.randn(n, generator=gen, device="cuda").bfloat16()
        ch = GpuBlockedChecker(W, 128, tree_height(n, 256, 8), generator=torch.Generator().manual_seed(40 + i))
        items.append((W, x, ch))

    def run(flags: int) -> list:
        a = GemvLaunch([items[0]], 256, verdicts=False)
        b = GemvLaunch([items[1]], 256, verdicts=False)
        for g in (a, b):
            for d in g._descs:
                d.flags = flags
        b.set_prior([a])
        a.set_prior([b])
        for _ in range(2):
            a.launch()
            b.launch()
        b.ys[0][300] += 1.0  # a fault in block 2 of b's output, planted after b ran
        a.launch()  # decides b's checks
        torch.cuda.synchronize()
        return [(r.passed.clone(), r.rho.clone(), r.tau.clone()) for g in (a, b) for r in g.results]

    settled, plain = run(_lib.PCK_CHECK_BANK_SETTLED), run(0)
    for (p1, r1, t1), (p0, r0, t0) in zip(settled, plain, strict=True):
        assert torch.equal(p1, p0) and torch.equal(r1, r0) and torch.equal(t1, t0)
    assert bool(settled[0][0].all())
    assert not bool(settled[1][0][0, 2]) and int(settled[1][0].sum()) == settled[1][0].numel() - 1
    with pytest.raises(RuntimeError, match="flags"):
        run(0x2)
