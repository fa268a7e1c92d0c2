"""The entry points as PyTorch custom operators (torch.ops.pck): registered with schemas
that name the scratch they write, traceable without a GPU through their fake
implementations (shapes and dtypes of every output), and on the GPU equal to the direct
C-ABI calls, under torch.compile and torch.library.opcheck."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import pck.cuda  # noqa: F401  (registers the operators)
from pck.cuda import ops


def test_every_operator_is_registered_with_its_mutations() -> None:
    for name in ops.OPS:
        op = getattr(torch.ops.pck, name).default
        schema = str(op._schema)
        writes = "partial_cx" in schema
        assert ("!)" in schema) == writes, schema
        assert writes == (name in ("blocked_check", "gemv_checked", "gemv_tc_checked")), name


def _fake_cuda(*shape, dtype):
    return torch.empty(shape, dtype=dtype, device="cuda")


def test_a_checked_decode_step_traces_without_a_gpu() -> None:
    """make_fx over fake CUDA tensors: every operator is one node, outputs shaped as the
    kernels write them."""
    m, n, batch, K, nb, seg, vocab = 1024, 4096, 4, 2, 8, 3, 1000

    def step(W, X, c, a, r, pcx, ps, logits, tokens, Q):
        y, passed, rho, tau = torch.ops.pck.gemv_checked(W, X, c, a, r, pcx, ps, 1e-3, 1e-12, 1e-40, 256)
        Y = torch.ops.pck.gemv_tc(W, X)
        Z = torch.ops.pck.gemv_fp8(Q, X, 256)
        ok, above, mass = torch.ops.pck.member_check(logits, tokens, None, None, None, 1e-4)
        cc, aa = torch.ops.pck.bank_build(W, r, 128, K, 1.0)
        return y, passed, rho, tau, Y, Z, ok, above, mass, cc, aa

    with FakeTensorMode():
        args = (_fake_cuda(m, n, dtype=torch.bfloat16), _fake_cuda(batch, n, dtype=torch.bfloat16),
                _fake_cuda(K, nb, n, dtype=torch.float32), _fake_cuda(nb, n, dtype=torch.bfloat16),
                _fake_cuda(K, nb, 128, dtype=torch.int8), _fake_cuda(batch, K, nb, seg, dtype=torch.float64),
                _fake_cuda(batch, nb, seg, dtype=torch.float64), _fake_cuda(batch, vocab, dtype=torch.float32),
                _fake_cuda(batch, dtype=torch.int64), _fake_cuda(m, n, dtype=torch.float8_e4m3fn))  # fmt: skip
        gm = make_fx(step, tracing_mode="fake")(*args)
        outs = gm(*args)
    targets = [str(nd.target) for nd in gm.graph.nodes if nd.op == "call_function"]
    for name in ("gemv_checked", "gemv_tc", "gemv_fp8", "member_check", "bank_build"):
        assert any(f"pck.{name}" in t for t in targets), (name, targets)
    y, passed, rho, tau, Y, Z, ok, above, mass, cc, aa = outs
    assert y.shape == (batch, m) and y.dtype == torch.float32
    assert passed.shape == (batch, K, nb) and passed.dtype == torch.bool and rho.dtype == torch.float64
    assert Y.shape == (batch, m) and Z.shape == (batch, m)
    assert ok.shape == (batch,) and above.dtype == torch.int64 and mass.dtype == torch.float64
    assert cc.shape == (K, m // 128, n) and aa.dtype == torch.bfloat16


def test_cpu_tensors_are_rejected_with_the_reference_wording() -> None:
    W = torch.zeros(128, 64, dtype=torch.bfloat16)
    x = torch.zeros(64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        torch.ops.pck.gemv_coalesced(W, x, 256)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_operators_on_the_gpu_match_the_direct_calls_and_compile() -> None:
    from pck.cuda import GpuBlockedChecker, gemv_tc, tc_height
    from pck.cuda._ext import extension

    gen = torch.Generator(device="cuda").manual_seed(3)
    W = (torch.randn(1024, 4096, generator=gen, device="cuda") * 0.02).bfloat16()
    x = torch.randn(4096, generator=gen, device="cuda").bfloat16()
    X = torch.randn(64, 4096, generator=gen, device="cuda").bfloat16()
    direct = extension().gemv_coalesced(W, x, 256)
    assert torch.equal(torch.ops.pck.gemv_coalesced(W, x, 256), direct)

    @torch.compile(fullgraph=True)
    def fn(W, x, X):
        return torch.ops.pck.gemv_coalesced(W, x, 256) * 2.0, torch.ops.pck.gemv_tc(W, X)

    y2, Y = fn(W, x, X)
    assert torch.equal(y2, direct * 2.0) and torch.equal(Y, gemv_tc(W, X))
    torch.library.opcheck(torch.ops.pck.gemv_coalesced.default, (W, x, 256))
    torch.library.opcheck(torch.ops.pck.gemv_tc.default, (W, X))
    ch = GpuBlockedChecker(W, 128, tc_height(4096), checks=1, generator=torch.Generator().manual_seed(1))
    pcx, ps = ch.scratch(64)
    torch.library.opcheck(torch.ops.pck.gemv_tc_checked.default,
                          (W, X, ch.c, ch.a, ch.r, pcx, ps, ch.coef, ch.geps, ch.tau_floor))  # fmt: skip
