"""The CPU oracle against golden vectors frozen from the reference's own code
(tests/golden/make_golden.py). CPU only."""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import checker as ochk
from oracle import fp as ofp
from oracle import gemv as ogemv
from oracle import member as omember
from oracle import sampling as osamp
from oracle.faults import flip_bit, sharded_topk
from tests.golden import inputs

GOLDEN = Path(__file__).parent / "golden"


def npz(name: str):
    return np.load(GOLDEN / f"{name}.npz")


FP = json.loads((GOLDEN / "fp.json").read_text())


# -- constants ------------------------------------------------------------------------------
def test_tree_height_matches_reference() -> None:
    for n, t, v, h in FP["tree_height"]:
        assert ofp.tree_height(n, t, v) == h, (n, t, v)
    assert ofp.tree_height(4096, 256, 8) == 23 and ofp.tree_height(4100, 256, 8) == 31


@pytest.mark.parametrize("key", ["gamma", "sum_up_factor", "softmax_eps"])
def test_constants_match_reference(key: str) -> None:
    fn = {"gamma": ofp.gamma, "sum_up_factor": ofp.sum_up_factor, "softmax_eps": ofp.softmax_eps}[key]
    for arg, want in FP[key]:
        assert fn(arg) == want


def test_gamma64_softmax_zmax_member_eps() -> None:
    for k, want in FP["gamma64"]:
        assert ofp.gamma(k, ofp.U64) == want
    for v, z, want in FP["softmax_eps_z"]:
        assert ofp.softmax_eps(v, z) == want
    for v, want in FP["member_eps"]:
        assert omember.member_eps(v) == want
    for v, want in FP["member_eps32"]:
        assert omember.member_eps32(v) == want


def test_bf16_and_round_up_f32_known_values() -> None:
    for v, want in FP["bf16"]:
        got = float(ofp.bf16(np.float32(v)))
        assert got == want or (math.isinf(got) and math.isinf(want))
    for v, want in FP["round_up_f32"]:
        assert float(ofp.round_up_f32([v])[0]) == want


def test_gpu_checker_host_constants_match_reference() -> None:
    for n, block, h, checks, segs, segments, coef, geps, floor in FP["gpu_checker_constants"]:
        want_segments = segments
        got_segments = segs if segs is not None else ochk.default_segments(n, checks, 2, 148)
        assert got_segments == want_segments
        assert ochk.host_constants(n, block, h, want_segments) == (coef, geps, floor)


# -- GEMV models ----------------------------------------------------------------------------
GEMV_CASES = [
    (1, 1, 32), (3, 5, 64), (7, 100, 32), (64, 1000, 32), (5, 17, 1024), (33, 4096, 128),
    (256, 4096, 256), (256, 4100, 256), (16, 14336, 512), (128, 4096, 1024), (9, 77, 64),
]  # fmt: skip


@pytest.mark.parametrize(("m", "n", "t"), GEMV_CASES)
def test_gemv_models_match_reference(m: int, n: int, t: int) -> None:
    g = npz("gemv")
    key = f"{m}x{n}_t{t}"
    W, x = inputs.numpy_problem(m, n, seed=m * n + t)
    assert inputs.digest(W, x) == str(g[f"digest_{key}"])
    if f"W_{key}" in g:
        np.testing.assert_array_equal(inputs.bits16(W), g[f"W_{key}"])
    y = ogemv.emulate_gemv_coalesced(W, x, t)
    np.testing.assert_array_equal(y.view(np.uint32), g[f"coalesced_{key}"])
    np.testing.assert_array_equal(ogemv.emulate_gemv(W, x, t).view(np.uint32), g[f"naive_{key}"])
    yc = ogemv.gemv_coalesced_c(inputs.bits16(W), inputs.bits16(x), t, 8)
    np.testing.assert_array_equal(yc.view(np.uint32), g[f"coalesced_{key}"])


def test_naive_small_threads_and_signed_zero_match_reference() -> None:
    g = npz("gemv")
    for t in (1, 2, 4, 16, 32, 256):
        W, x = inputs.numpy_problem(9, 77, seed=t)
        np.testing.assert_array_equal(ogemv.emulate_gemv(W, x, t).view(np.uint32), g[f"naive_small_t{t}"])
    Wz, xz = np.zeros((2, 64), dtype=np.float32), -np.ones(64, dtype=np.float32)
    for t in (32, 64):
        np.testing.assert_array_equal(
            ogemv.emulate_gemv_coalesced(Wz, xz, t).view(np.uint32), g[f"signed_zero_coalesced_t{t}"]
        )
        np.testing.assert_array_equal(ogemv.emulate_gemv(Wz, xz, t).view(np.uint32), g[f"signed_zero_naive_t{t}"])
        yc = ogemv.gemv_coalesced_c(inputs.bits16(Wz), inputs.bits16(xz), t, 8)
        np.testing.assert_array_equal(yc.view(np.uint32), g[f"signed_zero_coalesced_t{t}"])


def test_planted_shortcuts_match_reference() -> None:
    g = npz("gemv")
    W, x = inputs.numpy_problem(512, 2048, seed=2)
    for name, kw in (("legit", {}), ("drop_tail4", {"drop_tail": 4}), ("acc_bf16", {"acc_bf16": True}),
                     ("partial_bf16", {"partial_bf16": True})):  # fmt: skip
        np.testing.assert_array_equal(ogemv.emulate_gemv(W, x, 128, **kw).view(np.uint32), g[f"exploit_{name}"])


FP8_CASES = [(1, 1, 32), (3, 5, 64), (7, 100, 32), (5, 17, 1024), (33, 4096, 128), (256, 4100, 256),
             (64, 14336, 256)]  # fmt: skip


@pytest.mark.parametrize(("m", "n", "t"), FP8_CASES)
def test_fp8_model_matches_reference(m: int, n: int, t: int) -> None:
    g = npz("fp8")
    key = f"{m}x{n}_t{t}"
    W, x = inputs.torch_problem(m, n, seed=m * n + t)
    Q, s = inputs.quantize_fp8_cpu(W)
    assert inputs.digest(Q.view(torch.uint8).numpy(), x.float().numpy()) == str(g[f"digest_{key}"])
    np.testing.assert_array_equal(s.numpy(), g[f"s_{key}"])
    z = ogemv.emulate_gemv_coalesced(Q.float().numpy(), x.float().numpy(), t, vec=16)
    np.testing.assert_array_equal(z.view(np.uint32), g[f"z_{key}"])
    zc = ogemv.gemv_coalesced_c(Q.view(torch.uint8).numpy(), inputs.bits16(x.float().numpy()), t, 16,
                                ogemv.WEIGHT_E4M3)  # fmt: skip
    np.testing.assert_array_equal(zc.view(np.uint32), g[f"z_{key}"])


def test_fp8_bit_patterns_match_reference() -> None:
    g = npz("fp8")
    for seed in range(6):
        Q, x = inputs.fp8_bit_patterns(24, 600, seed)
        assert inputs.digest(Q.view(torch.uint8).numpy(), x.float().numpy()) == str(g[f"patterns_digest_{seed}"])
        zc = ogemv.gemv_coalesced_c(Q.view(torch.uint8).numpy(), inputs.bits16(x.float().numpy()), 64, 16,
                                    ogemv.WEIGHT_E4M3)  # fmt: skip
        np.testing.assert_array_equal(zc.view(np.uint32), g[f"patterns_z_{seed}"])


# -- configuration 1 and the checker bank ----------------------------------------------------
def test_config1_output_and_bank_match_reference() -> None:
    g = npz("config1")
    gen = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 4096, generator=gen) * 0.02).bfloat16()
    x = torch.randn(4096, generator=gen).bfloat16()
    W32, x32 = W.float().numpy(), x.float().numpy()
    assert inputs.digest(W32, x32) == str(g["digest"])
    y = ogemv.gemv_coalesced_c(inputs.bits16(W32), inputs.bits16(x32), 256, 8)
    np.testing.assert_array_equal(y.view(np.uint32), g["y"])
    bank = ochk.gpu_bank(W, 128, ofp.tree_height(4096, 256, 8), 1, gen, 8)
    np.testing.assert_array_equal(bank["r"].numpy(), g["r"])
    assert inputs.digest(bank["c"].numpy()) == str(g["c_digest"])
    assert inputs.digest(bank["a"].view(torch.int16).numpy()) == str(g["a_digest"])
    assert [bank["coef"], bank["geps"], bank["tau_floor"], bank["segments"]] == list(g["consts"])


def test_config1_cpu_checker_verdicts_match_reference() -> None:
    g = npz("config1")
    gen = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 4096, generator=gen) * 0.02).bfloat16()
    x = torch.randn(4096, generator=gen).bfloat16()
    W32, x32 = W.float().numpy(), x.float().numpy()
    y = ogemv.gemv_coalesced_c(inputs.bits16(W32), inputs.bits16(x32), 256, 8)
    h = ofp.tree_height(4096, 256, 8)
    planted = {
        "honest": y,
        "drop_tail64": ogemv.gemv_coalesced_c(
            inputs.bits16(np.where(np.arange(4096) >= 4032, 0, W32).astype(np.float32)), inputs.bits16(x32), 256, 8
        ),
        "bf16_output": ofp.bf16(y),
        "exponent_flip": flip_bit(y, 777, 27),
        "sign_flip": flip_bit(y, 1234, 31),
    }
    bank = ochk.WeightBank(W32, 128)
    for name, yy in planted.items():
        assert inputs.digest(yy) == str(g[f"planted_digest_{name}"]), name
        chk = ochk.BlockedChecker(W32, x32, 128, h, bank)
        np.testing.assert_array_equal(chk.verdict(yy, np.random.default_rng(7), checks=4), g[f"cpu_verdict_{name}"])
    assert g["cpu_verdict_honest"].all() and not g["cpu_verdict_drop_tail64"].all()


def test_small_bank_matches_reference_bitwise() -> None:
    g = npz("bank_small")
    Wn, xn = inputs.numpy_problem(256, 1000, seed=1)
    assert inputs.digest(Wn, xn) == str(g["digest"])
    bank = ochk.gpu_bank(torch.from_numpy(Wn).bfloat16(), 32, 23, 4, torch.Generator().manual_seed(1), 3)
    np.testing.assert_array_equal(bank["r"].numpy(), g["r"])
    np.testing.assert_array_equal(bank["c"].numpy().view(np.uint32), g["c"].view(np.uint32))
    np.testing.assert_array_equal(bank["a"].view(torch.int16).numpy(), g["a"])
    assert [bank["coef"], bank["geps"], bank["tau_floor"], bank["segments"]] == list(g["consts"])


def test_round_up_bf16_matches_reference() -> None:
    ref = json.loads((GOLDEN / "round_up_bf16.json").read_text())
    got = ochk.round_up_bf16(torch.tensor(ref["in"], dtype=torch.float64)).float().tolist()
    assert got == ref["out"]


# -- membership -------------------------------------------------------------------------------
def _assert_members(name: str, out: dict, g, vocab: int, compare_member: bool = True) -> None:
    np.testing.assert_array_equal(out["ok"], g[f"{name}_ok"])
    np.testing.assert_array_equal(out["above"], g[f"{name}_above"])
    ok = g[f"{name}_ok"]
    mass_ref = g[f"{name}_mass"]
    tol = omember.member_eps32(vocab)
    sel = ok & np.isfinite(mass_ref)
    assert np.all(np.abs(out["mass_above"][sel] - mass_ref[sel]) <= tol)
    if compare_member:
        np.testing.assert_array_equal(g[f"{name}_member_ok"], ok)


def test_members_ties_match_reference() -> None:
    g = npz("member")
    logits, tokens, top_k, top_p, greedy = inputs.member_case_ties()
    out = omember.check_members(logits, tokens, top_k, top_p, greedy)
    _assert_members("ties", out, g, 500)
    for i in range(64):
        k = None if top_k[i] == 500 else int(top_k[i])
        p = None if top_p[i] == 1.0 else float(top_p[i])
        v = omember.check_member(logits[i], int(tokens[i]), k, p, greedy=bool(greedy[i]))
        assert v.ok == bool(g["ties_member_ok"][i]) and v.above == int(g["ties_member_above"][i])


def test_members_kth_ties_and_wide_match_reference() -> None:
    g = npz("member")
    logits, tokens, top_k, top_p = inputs.member_case_kth_ties()
    _assert_members("kth_ties", omember.check_members(logits, tokens, top_k, top_p), g, 400)
    logits, tokens = inputs.member_case_wide()
    _assert_members("wide", omember.check_members(logits, tokens, top_p=np.full(16, 0.99)), g, 5000)


def test_members_bad_ids_and_lm_head_match_reference() -> None:
    g = npz("member")
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((4, 50)).astype(np.float32)
    tokens = np.array([-1, 50, 10_000, int(logits[3].argmax())])
    out = omember.check_members(logits, tokens, np.array([5, 5, 5, 20]), np.full(4, 0.9))
    np.testing.assert_array_equal(out["ok"], g["bad_ids_ok"])
    np.testing.assert_array_equal(out["above"], g["bad_ids_above"])
    lg, tok, tk, tp, faulty = inputs.member_case_lm_head(64, 128256, seed=5)
    assert inputs.digest(lg.numpy(), tok.numpy()) == str(g["lm_head_digest"])
    out = omember.check_members(lg.numpy(), tok.numpy(), tk.numpy(), tp.numpy())
    np.testing.assert_array_equal(out["ok"], g["lm_head_ok"])
    np.testing.assert_array_equal(out["above"], g["lm_head_above"])
    sel = g["lm_head_ok"]
    assert np.all(np.abs(out["mass_above"][sel] - g["lm_head_mass"][sel]) <= omember.member_eps32(128256))
    np.testing.assert_array_equal(~g["lm_head_ok"], g["lm_head_faulty"])  # every fault caught, nothing else


# -- sampling set checks -----------------------------------------------------------------------
def test_sampling_checks_match_reference() -> None:
    g = npz("sampling")
    for seed in range(5):
        lg = inputs.sampling_logits(8, 2000, seed, ties=True)
        sel = g[f"swap_sel_{seed}"]
        got = [osamp.check_topk(lg[b], sel[b], 20) for b in range(8)]
        np.testing.assert_array_equal(got, g[f"swap_verdict_{seed}"])
    lg = inputs.sampling_logits(8, 500, 11)
    for delta in (-1, 0, 1):
        sels = g[f"topp_delta{delta}_sel"]
        got = [osamp.check_topp(lg[b], sels[b][sels[b] >= 0], 0.8, tol=0.0) for b in range(8)]
        np.testing.assert_array_equal(got, g[f"topp_delta{delta}_verdict"])
    lg = inputs.sampling_logits(8, 4096, 3)
    lg[0, :16] = 100.0 + np.arange(16, dtype=np.float32)
    for per_shard in (4, 16):
        sel = np.stack([sharded_topk(lg[b], 16, 8, per_shard) for b in range(8)])
        np.testing.assert_array_equal(sel, g[f"sharded_{per_shard}_sel"])
        got = [osamp.check_topk(lg[b], sel[b], 16) for b in range(8)]
        np.testing.assert_array_equal(got, g[f"sharded_{per_shard}_verdict"])
