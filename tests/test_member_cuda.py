"""The membership kernel against the reference's outputs (golden fixtures of
src/pck/member.py:check_members) and the CPU oracle: `ok` and `above` identical, `mass_above`
within the two computations' error bounds (2 member_eps32)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import member as omember
from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

GOLDEN = np.load(Path(__file__).parent / "golden" / "member.npz")


def run(logits, tokens, top_k=None, top_p=None, greedy=None, dtype=torch.float32):
    from pck.member import check_members

    lg = torch.as_tensor(logits).to(dtype).cuda()
    dev = lambda v: None if v is None else torch.as_tensor(np.asarray(v)).cuda()  # noqa: E731
    out = check_members(lg, dev(tokens), dev(top_k), dev(top_p), dev(greedy))
    return {k: v.cpu().numpy() for k, v in out.items()}


def assert_like(out: dict, ok, above, mass, vocab: int, factor: float = 2.0, accepted_only: bool = False) -> None:
    """``accepted_only``: compare the masses of accepted rows only. The reference's fast
    branch (every row with a top-k) leaves out of A the kept tokens tied at the k-th logit
    beyond its top-`max k` list, which differs from the definition only on rows that top-k
    already rejects (ok and above are unaffected); the oracle follows the definition."""
    np.testing.assert_array_equal(out["ok"], ok)
    np.testing.assert_array_equal(out["above"], above)
    mass = np.asarray(mass)
    both = np.isfinite(mass) & np.isfinite(out["mass_above"])
    if accepted_only:
        both &= np.asarray(ok)
    else:
        np.testing.assert_array_equal(np.isfinite(out["mass_above"]), np.isfinite(mass))
    assert np.all(np.abs(out["mass_above"][both] - mass[both]) <= factor * omember.member_eps32(vocab))


def test_golden_ties() -> None:
    logits, tokens, top_k, top_p, greedy = inputs.member_case_ties()
    out = run(logits, tokens, top_k, top_p, greedy)
    assert_like(out, GOLDEN["ties_ok"], GOLDEN["ties_above"], GOLDEN["ties_mass"], 500, accepted_only=True)


def test_golden_kth_ties_and_wide() -> None:
    logits, tokens, top_k, top_p = inputs.member_case_kth_ties()
    out = run(logits, tokens, top_k, top_p)
    assert_like(out, GOLDEN["kth_ties_ok"], GOLDEN["kth_ties_above"], GOLDEN["kth_ties_mass"], 400,
                accepted_only=True)  # fmt: skip
    want = omember.check_members(logits, tokens, top_k, top_p)
    assert_like(out, want["ok"], want["above"], want["mass_above"], 400)
    logits, tokens = inputs.member_case_wide()
    out = run(logits, tokens, top_p=np.full(16, 0.99))
    assert_like(out, GOLDEN["wide_ok"], GOLDEN["wide_above"], GOLDEN["wide_mass"], 5000, accepted_only=True)


def test_golden_bad_ids() -> None:
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((4, 50)).astype(np.float32)
    tokens = np.array([-1, 50, 10_000, int(logits[3].argmax())])
    out = run(logits, tokens, np.array([5, 5, 5, 20]), np.full(4, 0.9))
    np.testing.assert_array_equal(out["ok"], GOLDEN["bad_ids_ok"])
    np.testing.assert_array_equal(out["above"], GOLDEN["bad_ids_above"])


def test_golden_lm_head_every_fault_caught() -> None:
    """Config-5 batch: 64 rows of 128,256 logits, top-k 50, top-p 0.9, 1% argmin tokens."""
    lg, tok, tk, tp, faulty = inputs.member_case_lm_head(64, 128256, seed=5)
    out = run(lg, tok, tk, tp)
    assert_like(out, GOLDEN["lm_head_ok"], GOLDEN["lm_head_above"], GOLDEN["lm_head_mass"], 128256,
                accepted_only=True)  # fmt: skip
    np.testing.assert_array_equal(~out["ok"], faulty.numpy())


def random_case(rng, rows: int, vocab: int, ties: bool):
    logits = (rng.standard_normal((rows, vocab)) * rng.choice([0.5, 3.0, 30.0])).astype(np.float32)
    if ties:
        logits[:, : max(1, vocab // 10)] = logits.max()
    tokens = rng.integers(-2, vocab + 2, rows)
    order = np.argsort(-logits, axis=1)
    near = rng.random(rows) < 0.7
    tokens[near] = order[near, rng.integers(0, max(1, min(vocab, 30)), near.sum())]
    top_k = rng.choice([1, 2, 5, 50, vocab, vocab + 5, max(1, vocab // 2)], rows)
    top_p = rng.choice([0.1, 0.5, 0.9, 0.999, 1.0, 1.5], rows)
    greedy = rng.random(rows) < 0.2
    return logits, tokens, top_k, top_p, greedy


@pytest.mark.parametrize("vocab", [1, 2, 7, 100, 1000, 1500, 5000, 40000])
@pytest.mark.parametrize("ties", [False, True])
def test_matches_oracle(vocab: int, ties: bool) -> None:
    rng = np.random.default_rng(vocab * 2 + ties)
    logits, tokens, top_k, top_p, greedy = random_case(rng, 12, vocab, ties)
    want = omember.check_members(logits, tokens, top_k, top_p, greedy)
    out = run(logits, tokens, top_k, top_p, greedy)
    assert_like(out, want["ok"], want["above"], want["mass_above"], vocab)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_precision_logits_match_oracle(dtype) -> None:
    rng = np.random.default_rng(7)
    logits, tokens, top_k, top_p, greedy = random_case(rng, 16, 3000, False)
    lg = torch.tensor(logits).to(dtype)
    want = omember.check_members(lg.float().numpy(), tokens, top_k, top_p, greedy)
    out = run(lg, tokens, top_k, top_p, greedy, dtype=dtype)
    assert_like(out, want["ok"], want["above"], want["mass_above"], 3000)


def test_optional_arguments_absent() -> None:
    rng = np.random.default_rng(8)
    logits, tokens, top_k, top_p, _ = random_case(rng, 10, 600, False)
    for tk, tp in ((None, None), (top_k, None), (None, top_p)):
        want = omember.check_members(logits, tokens, tk, tp)
        out = run(logits, tokens, tk, tp)
        assert_like(out, want["ok"], want["above"], want["mass_above"], 600)
        if tp is None:
            assert not out["mass_above"].any()


def test_nan_inf_and_large_k_fallbacks() -> None:
    """NaN rows reject with NaN mass; -inf logits; k above the CTA's thread count and rows
    whose candidates overflow shared memory (all logits tied) take the whole-row select."""
    rng = np.random.default_rng(9)
    vocab = 20000
    logits = (rng.standard_normal((6, vocab)) * 3).astype(np.float32)
    logits[0, 17] = np.nan
    logits[1, ::3] = -np.inf
    logits[2] = 1.25  # every logit tied: all are candidates
    logits[3, : vocab // 2] = 4.0  # half tied at the top
    tokens = np.array([5, int(np.argmax(logits[1])), 3, 2, int(np.argsort(-logits[4])[1500]), 0])
    top_k = np.array([50, 50, 10, 100, 3000, 1025])
    top_p = np.array([0.9, 0.9, 0.5, 0.7, 0.95, 0.8])
    want = omember.check_members(logits, tokens, top_k, top_p)
    out = run(logits, tokens, top_k, top_p)
    assert_like(out, want["ok"], want["above"], want["mass_above"], vocab)
    assert not out["ok"][0] and np.isnan(out["mass_above"][0])


def test_strided_rows_and_empty_batch() -> None:
    from pck.member import check_members

    rng = np.random.default_rng(10)
    big = torch.tensor((rng.standard_normal((8, 1200)) * 3).astype(np.float32)).cuda()
    view = big[:, 100:1100]  # row stride 1200, 1000 logits per row
    tokens = view.argmax(dim=1)
    out = check_members(view, tokens, torch.full((8,), 40).cuda(), torch.full((8,), 0.9).cuda())
    want = omember.check_members(view.cpu().numpy(), tokens.cpu().numpy(), np.full(8, 40), np.full(8, 0.9))
    np.testing.assert_array_equal(out["ok"].cpu().numpy(), want["ok"])
    empty = check_members(torch.empty((0, 10)).cuda(), torch.empty(0, dtype=torch.int64).cuda())
    assert empty["ok"].shape == (0,)


def test_rejects_host_tensors_and_bad_shapes() -> None:
    from pck.member import check_members

    with pytest.raises(RuntimeError, match="CUDA"):
        check_members(torch.zeros(2, 5), torch.zeros(2, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="one value per row"):
        check_members(torch.zeros(2, 5).cuda(), torch.zeros(3, dtype=torch.int64).cuda())
