"""E4M3 GEMV: bit-exact with the reference's vec-16 model, checked against its FP8 weights
(the reference's tests/gpu/test_gemv_fp8.py)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle.gemv import WEIGHT_E4M3, gemv_coalesced_c
from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

GOLDEN = np.load(Path(__file__).parent / "golden" / "fp8.npz")
CASES = [(1, 1, 32), (3, 5, 64), (7, 100, 32), (5, 17, 1024), (33, 4096, 128), (256, 4100, 256),
         (64, 14336, 256)]  # fmt: skip


def c_model(Q: torch.Tensor, x: torch.Tensor, threads: int) -> np.ndarray:
    return gemv_coalesced_c(Q.view(torch.uint8).cpu().numpy(), x.view(torch.uint16).cpu().numpy(), threads, 16,
                            WEIGHT_E4M3)  # fmt: skip


@pytest.mark.parametrize(("m", "n", "t"), CASES)
def test_matches_reference_golden(m: int, n: int, t: int) -> None:
    """The golden z was computed from the reference's CPU quantisation; torch's GPU
    division may round the scales differently, so the same CPU-quantised Q is fed here."""
    from pck.cuda import gemv_fp8

    W, x = inputs.torch_problem(m, n, seed=m * n + t)
    Q, s = inputs.quantize_fp8_cpu(W)
    np.testing.assert_array_equal(s.numpy(), GOLDEN[f"s_{m}x{n}_t{t}"])
    z = gemv_fp8(Q.cuda(), x.cuda(), t)
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), GOLDEN[f"z_{m}x{n}_t{t}"])


def test_gpu_quantisation_feeds_a_bit_exact_gemv() -> None:
    from pck.cuda import gemv_fp8, quantize_fp8

    W, x = inputs.torch_problem(256, 4096, seed=77)
    Q, _ = quantize_fp8(W.cuda())
    z = gemv_fp8(Q, x.cuda(), 256)
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), c_model(Q, x, 256).view(np.uint32))


@pytest.mark.parametrize("seed", range(6))
def test_every_e4m3_pattern_matches_reference(seed: int) -> None:
    from pck.cuda import gemv_fp8

    Q, x = inputs.fp8_bit_patterns(24, 600, seed)
    z = gemv_fp8(Q.cuda(), x.cuda(), 64)
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), GOLDEN[f"patterns_z_{seed}"])


@settings(max_examples=40, deadline=None)
@given(st.integers(1, 32), st.sampled_from([16, 32, 256, 4096, 600, 1]), st.sampled_from([32, 64, 128, 256]),
       st.integers(0, 2**31 - 1))  # fmt: skip
def test_random_patterns_match_oracle(m: int, n: int, threads: int, seed: int) -> None:
    from pck.cuda import gemv_fp8

    Q, x = inputs.fp8_bit_patterns(m, n, seed)
    z = gemv_fp8(Q.cuda(), x.cuda(), threads)
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), c_model(Q, x, threads).view(np.uint32))


def test_huge_activations_take_the_exact_product_path() -> None:
    """|x| near the binary32 limit: products overflow, so the kernel must not fuse them."""
    from pck.cuda import gemv_fp8

    Q, x = inputs.fp8_bit_patterns(64, 4096, 11)
    x = x.float()
    x[5] = 2.0**121  # one huge activation: rows with a nonzero weight there overflow
    x[4000] = -(2.0**120)
    x = x.bfloat16()
    Q = Q.clone()
    Q.view(torch.uint8)[::2, 4000] = 0  # even rows: only the +huge column, no inf - inf
    z = gemv_fp8(Q.cuda(), x.cuda(), 256).cpu().numpy()
    ref = c_model(Q, x, 256)
    # NaN results (inf - inf) carry the platform's NaN encoding; everything else is bitwise
    np.testing.assert_array_equal(np.isnan(z), np.isnan(ref))
    keep = ~np.isnan(ref)
    np.testing.assert_array_equal(z[keep].view(np.uint32), ref[keep].view(np.uint32))
    assert keep.any()


@pytest.mark.parametrize(("m", "n"), [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_decode_shapes_match_c_oracle(m: int, n: int) -> None:
    from pck.cuda import gemv_fp8, quantize_fp8

    W, x = inputs.torch_problem(m, n, seed=m + 3 * n)
    Q, _ = quantize_fp8(W.cuda())
    z = gemv_fp8(Q, x.cuda(), 256)
    np.testing.assert_array_equal(z.cpu().numpy().view(np.uint32), c_model(Q, x, 256).view(np.uint32))


def test_unaligned_pointer_uses_scalar_path() -> None:
    from pck.cuda import gemv_fp8, quantize_fp8

    m, n, threads = 8, 4096, 128
    W, x = inputs.torch_problem(m, n, seed=3)
    Q = quantize_fp8(W.cuda())[0]
    flat = torch.zeros(m * n + 1, dtype=torch.uint8, device="cuda")
    flat[1:] = Q.view(torch.uint8).flatten()
    view = flat[1:].view(torch.float8_e4m3fn).view(m, n)
    assert view.is_contiguous() and view.data_ptr() % 16 != 0
    assert torch.equal(gemv_fp8(view, x.cuda(), threads), gemv_fp8(Q, x.cuda(), threads))


def test_quantize_fp8_scales_rows() -> None:
    from pck.cuda import quantize_fp8

    W, _ = inputs.torch_problem(16, 300, seed=1)
    W = W.cuda()
    W[3] = 0
    Q, s = quantize_fp8(W)
    assert Q.dtype == torch.float8_e4m3fn and s.shape == (16,)
    assert s[3] == 1 and not Q[3].float().any()
    assert torch.allclose(Q.float().abs().amax(dim=1)[s != 1], torch.tensor(448.0).cuda())
    assert (s[:, None] * Q.float() - W.float()).norm() / W.float().norm() < 0.05


def test_rejects_bf16_weights() -> None:
    from pck.cuda import gemv_fp8

    W, x = inputs.torch_problem(4, 32, seed=0)
    with pytest.raises(RuntimeError, match="Float8_e4m3fn"):
        gemv_fp8(W.cuda(), x.cuda())


def checker_for(Q: torch.Tensor, threads: int):
    from pck.cuda import GpuBlockedChecker
    from pck.fp import tree_height

    return GpuBlockedChecker(Q.to(torch.bfloat16), 128, tree_height(Q.shape[1], threads, 16), checks=8,
                             generator=torch.Generator().manual_seed(0))  # fmt: skip


def test_checker_passes_fp8_output() -> None:
    from pck.cuda import gemv_fp8, quantize_fp8

    W, _ = inputs.torch_problem(1024, 4096, seed=7)
    Q = quantize_fp8(W.cuda())[0]
    checker = checker_for(Q, 256)
    for seed in range(5):
        x = inputs.torch_problem(1, 4096, seed=100 + seed)[1].cuda()
        assert checker.verdict(x, gemv_fp8(Q, x, 256)).all()


def test_checker_catches_faults_in_fp8_output() -> None:
    from pck.cuda import gemv_fp8, quantize_fp8

    W, x = inputs.torch_problem(1024, 4096, seed=8)
    Q = quantize_fp8(W.cuda())[0]
    x = x.cuda()
    checker = checker_for(Q, 256)
    z = gemv_fp8(Q, x, 256)
    assert not checker.verdict(x, z.bfloat16().float()).all()
    flipped = z.clone()
    flipped.view(torch.int32)[5] ^= 1 << 30
    assert not checker.verdict(x, flipped)[0]
