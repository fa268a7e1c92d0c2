"""Config 5 on one GPU: the LM head W (128256, 4096) bfloat16 at decode batch 64 through the
checked tensor-core GEMV, then top-k 50 / top-p 0.9 sampling at temperature 1 and the fused
membership check of every sampled token, with 1% of the tokens replaced by the row's lowest
logit (src/pck/vllm_plugin.py:174-182).

  - every block of the honest logits passes its check;
  - every logit lies within the declared rounding bound of the tensor-core accumulation,
    |y - W x| <= gamma_h (|W| |x|) with h = tc_height(n), against a binary64 product;
  - the membership verdicts (`ok`, `above`) equal the oracle's (a CPU restatement of
    src/pck/member.py) row for row, masses within 2 member_eps32 + tol slack;
  - every planted token is rejected and no honest one is.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import member as omember
from oracle.fp import U32, gamma

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

VOCAB, N, BATCH = 128256, 4096, 64
# activations scaled so that the logits are ~N(0, 3^2): W ~ N(0, 0.02^2) over n = 4096
X_SCALE = 3.0 / (0.02 * N**0.5)


def lm_head_problem(vocab: int = VOCAB, batch: int = BATCH, seed: int = 0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    W = (torch.randn(vocab, N, generator=gen, device="cuda") * 0.02).bfloat16()
    X = (torch.randn(batch, N, generator=gen, device="cuda") * X_SCALE).bfloat16()
    return W, X


@pytest.fixture(scope="module")
def head():
    from pck.cuda.lm_head import CheckedLMHead

    W, X = lm_head_problem()
    h = CheckedLMHead(W, X, VOCAB, generator=torch.Generator().manual_seed(7))
    h.forward()
    torch.cuda.synchronize()
    return h


def test_logits_pass_and_stay_within_the_declared_bound(head) -> None:
    from pck.cuda import device_status, tc_height

    assert bool(head.passed.all())
    assert head.logits.shape == (BATCH, VOCAB)
    bound_factor = gamma(tc_height(N), U32)
    for r0 in range(0, VOCAB, 16384):  # binary64 reference in slices of the vocabulary
        Wd = head.W[r0 : r0 + 16384].double()
        Xd = head.X.double()
        exact = Xd @ Wd.T
        mag = Xd.abs() @ Wd.abs().T
        err = (head.logits[:, r0 : r0 + 16384].double() - exact).abs()
        assert bool((err <= bound_factor * mag).all())
        ratio = float((err / (bound_factor * mag).clamp(min=1e-300)).max())
        assert ratio < 0.5, f"observed error at {ratio:.3f} of the declared bound"
    std = float(head.logits.std())
    assert 2.5 < std < 3.5  # the config's logits ~ N(0, 3^2)
    assert device_status() == 0


def test_sampled_tokens_membership_matches_oracle_and_catches_planted(head) -> None:
    from pck.cuda.lm_head import TopKTopPSampler, membership
    from pck.member import member_eps32

    torch.manual_seed(11)
    sampler = TopKTopPSampler(BATCH, VOCAB, k=50, p=0.9, temperature=1.0, device=head.device, fault_rate=0.01)
    logits_np = head.logits.cpu().numpy()
    planted = caught = false_alarms = 0
    for step in range(30):
        tokens = sampler(head.logits)
        verdict = membership(head.logits, sampler)
        torch.cuda.synchronize()
        ok = verdict["ok"].cpu().numpy()
        injected = sampler.injected.cpu().numpy()
        planted += int(injected.sum())
        caught += int((~ok & injected).sum())
        false_alarms += int((~ok & ~injected).sum())
        if step < 4:  # row-for-row against the oracle on a few steps (each is 64 full rows)
            ref = omember.check_members(logits_np, tokens.cpu().numpy(), top_k=np.full(BATCH, 50),
                                        top_p=np.full(BATCH, 0.9), greedy=None, tol=1e-4)  # fmt: skip
            np.testing.assert_array_equal(ok, ref["ok"])
            np.testing.assert_array_equal(verdict["above"].cpu().numpy(), ref["above"])
            mass = verdict["mass_above"].cpu().numpy()
            acc = ref["ok"]
            assert np.all(np.abs(mass[acc] - ref["mass_above"][acc]) <= 2 * member_eps32(VOCAB))
    assert planted > 0, "the seeded draws planted nothing"
    assert caught == planted and false_alarms == 0


def test_sharded_rows_reassemble_bitwise_on_one_gpu(head) -> None:
    """The logits of the row shards of two, four and eight ranks, each computed on its own
    (what every rank computes), concatenate to the unsharded logits bit for bit: with
    full_k the tensor-core kernel's order does not depend on the shard (whole tiles, full K
    per tile)."""
    from pck.cuda import gemv_tc
    from pck.cuda.sharded import shard_rows

    for world in (2, 4, 8):
        parts = []
        for rank in range(world):
            sh = shard_rows(VOCAB, 128, world, rank)
            parts.append(gemv_tc(head.W[sh.row0 : sh.row1].contiguous(), head.X, full_k=True))
        full = torch.cat(parts, dim=-1)
        torch.cuda.synchronize()
        assert torch.equal(full.view(torch.int32), head.logits.view(torch.int32)), f"world {world}"


def test_sampler_kernel_draws_as_the_torch_sampler(head) -> None:
    """The fused sampler (`pck_sample_topk_topp`) against the torch sampler on the same logits
    and the same uniform draws: every kernel token is one of the row's k largest logits and
    inside the nucleus (probability mass before it, in descending order, below p, in binary64),
    nearly every row picks the same token (the binary32 running sums may differ on a draw that
    falls on a boundary), and the planted rows carry the row's argmin."""
    from pck.cuda.lm_head import TopKTopPSampler

    k, p = 50, 0.9
    ker = TopKTopPSampler(BATCH, VOCAB, k, p, 1.0, head.device, fault_rate=0.05)
    ref = TopKTopPSampler(BATCH, VOCAB, k, p, 1.0, head.device, fault_rate=0.05, impl="torch")
    logits = head.logits
    vals, idx = torch.topk(logits.double(), k, dim=-1)
    probs = torch.softmax(vals, dim=-1)
    before = torch.cumsum(probs, dim=-1) - probs
    argmin = logits.argmin(dim=-1)
    same = total = planted = 0
    for step in range(20):
        gen = torch.Generator(device=head.device).manual_seed(300 + step)
        draws = torch.rand(BATCH, generator=gen, device=head.device)
        faults = torch.rand(BATCH, generator=gen, device=head.device)
        for s in (ker, ref):
            s.draw.uniform_ = lambda d=draws, s=s: s.draw.copy_(d)  # noqa: B023 (fixed draws)
            s.fault_draw.uniform_ = lambda f=faults, s=s: s.fault_draw.copy_(f)  # noqa: B023
        t_ker = ker(logits).clone()
        inj = ker.injected.clone()
        t_ref = ref(logits).clone()
        assert torch.equal(inj, ref.injected)
        assert torch.equal(t_ker[inj], argmin[inj])
        planted += int(inj.sum())
        honest = ~inj
        pos = (idx == t_ker.unsqueeze(-1))
        assert bool(pos[honest].any(dim=-1).all()), "a token outside the top k"
        b = (before * pos).sum(dim=-1)
        assert bool((b[honest] < p).all()), "a token outside the nucleus"
        same += int((t_ker == t_ref)[honest].sum())
        total += int(honest.sum())
    assert planted > 0
    assert same >= 0.95 * total, f"{same} of {total} rows agree"
