"""The top-k / top-p set checker on the GPU against the reference's verdicts (golden
fixtures of src/pck/sampling.py) and the CPU oracle (the reference's tests/gpu/
test_sampling_cuda.py, restated)."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sampling as osamp
from oracle.faults import sharded_topk
from tests.golden import inputs

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

GOLDEN = np.load(Path(__file__).parent / "golden" / "sampling.npz")


def logits(rows: int, vocab: int, seed: int, scale: float = 3.0, ties: bool = False) -> torch.Tensor:
    return torch.from_numpy(inputs.sampling_logits(rows, vocab, seed, scale, ties)).cuda()


def test_golden_swaps_topp_off_by_one_and_sharded() -> None:
    from pck.cuda import check_topk_gpu, check_topp_gpu

    for seed in range(5):
        lg = logits(8, 2000, seed, ties=True)
        sel = torch.from_numpy(GOLDEN[f"swap_sel_{seed}"]).cuda()
        got = check_topk_gpu(lg, sel, 20).passed.cpu().numpy()
        np.testing.assert_array_equal(got, GOLDEN[f"swap_verdict_{seed}"])
    lg = logits(8, 500, 11)
    for delta in (-1, 0, 1):
        sels = GOLDEN[f"topp_delta{delta}_sel"]
        lengths = torch.tensor((sels >= 0).sum(axis=1), dtype=torch.int64).cuda()
        sel = torch.from_numpy(np.where(sels >= 0, sels, 0)).cuda()
        got = check_topp_gpu(lg, sel, lengths, 0.8, tol=0.0).passed.cpu().numpy()
        np.testing.assert_array_equal(got, GOLDEN[f"topp_delta{delta}_verdict"])
    lg = logits(8, 4096, 3)
    lg[0, :16] = 100.0 + torch.arange(16, dtype=torch.float32, device="cuda")
    for per_shard in (4, 16):
        sel = torch.from_numpy(GOLDEN[f"sharded_{per_shard}_sel"]).cuda()
        got = check_topk_gpu(lg, sel, 16).passed.cpu().numpy()
        np.testing.assert_array_equal(got, GOLDEN[f"sharded_{per_shard}_verdict"])


@pytest.mark.parametrize(("vocab", "k"), [(1, 1), (7, 3), (1000, 50), (4096, 1), (151_936, 40)])
@pytest.mark.parametrize("ties", [False, True])
def test_topk_sampler_passes_and_matches_oracle(vocab: int, k: int, ties: bool) -> None:
    from pck.cuda import check_topk_gpu, topk_sample

    lg = logits(8, vocab, seed=vocab + k, ties=ties)
    selected, token = topk_sample(lg, k, generator=torch.Generator("cuda").manual_seed(0))
    res = check_topk_gpu(lg, selected, k)
    assert res.passed.all()
    assert (selected == token[:, None]).any(dim=1).all()
    for b in range(8):
        assert osamp.check_topk(lg[b].cpu().numpy(), selected[b].cpu().numpy(), k)


@pytest.mark.parametrize("seed", range(4))
def test_random_swaps_match_oracle(seed: int) -> None:
    from pck.cuda import check_topk_gpu, topk_sample

    rows, vocab, k = 8, 3000, 25
    lg = logits(rows, vocab, seed=100 + seed, ties=True)
    sel = topk_sample(lg, k)[0].clone()
    rng = np.random.default_rng(seed)
    for b in range(rows):
        other = np.setdiff1d(np.arange(vocab), sel[b].cpu().numpy())
        sel[b, rng.integers(k)] = int(rng.choice(other))
    gpu = check_topk_gpu(lg, sel, k)
    cpu = [osamp.check_topk(lg[b].cpu().numpy(), sel[b].cpu().numpy(), k) for b in range(rows)]
    np.testing.assert_array_equal(gpu.passed.cpu().numpy(), cpu)
    for b in range(rows):  # the exact extremes
        a, s = lg[b].cpu().numpy(), sel[b].cpu().numpy()
        mask = np.zeros(vocab, dtype=bool)
        mask[s] = True
        assert gpu.min_selected[b].item() == a[mask].min() and gpu.max_rejected[b].item() == a[~mask].max()


def test_sharded_fault_is_caught_when_the_top_clusters() -> None:
    from pck.cuda import check_topk_gpu, sharded_topk_gpu

    lg = logits(4, 4096, seed=31)
    lg[:, :16] = 50.0 + torch.arange(16, dtype=torch.float32, device="cuda")  # all of the top in shard 0
    sel = sharded_topk_gpu(lg, 16, shards=8, per_shard=4)
    np.testing.assert_array_equal(sel.cpu().numpy(), np.stack([sharded_topk(r, 16, 8, 4) for r in lg.cpu().numpy()]))
    assert not check_topk_gpu(lg, sel, 16).passed.any()
    assert check_topk_gpu(lg, sharded_topk_gpu(lg, 16, shards=8, per_shard=16), 16).passed.all()


@pytest.mark.parametrize("fault", ["duplicate", "out_of_range", "negative", "nan", "short", "long"])
def test_malformed_or_nan_fails_only_its_row(fault: str) -> None:
    from pck.cuda import check_topk_gpu, topk_sample

    lg = logits(6, 777, seed=41)
    sel = topk_sample(lg, 10)[0].clone()
    k = 10
    if fault == "duplicate":
        sel[2, 3] = sel[2, 4]
    elif fault == "out_of_range":
        sel[2, 0] = 777
    elif fault == "negative":
        sel[2, 9] = -1
    elif fault == "nan":
        lg[2, 500] = float("nan")
    res = check_topk_gpu(lg, sel, k if fault not in ("short", "long") else (11 if fault == "short" else 9))
    want = [True] * 6 if fault not in ("short", "long") else [False] * 6
    if fault not in ("short", "long"):
        want[2] = False
    assert res.passed.cpu().tolist() == want


@pytest.mark.parametrize(("vocab", "p", "temp"), [(50, 0.5, 1.0), (1000, 0.9, 1.0), (32_000, 0.95, 0.7),
                                                  (151_936, 0.9, 1.3)])  # fmt: skip
def test_topp_sampler_passes_and_masses_match_oracle(vocab: int, p: float, temp: float) -> None:
    from pck.cuda import check_topp_gpu, topp_select

    lg = logits(4, vocab, seed=vocab)
    sel, lengths = topp_select(lg, p, temp)
    res = check_topp_gpu(lg, sel, lengths, p, temperature=temp, tol=1e-5)
    assert res.passed.all()
    for b in range(4):
        a = lg[b].cpu().numpy()
        s = sel[b, : lengths[b]].cpu().numpy()
        assert osamp.check_topp(a, s, p, temperature=temp, tol=1e-5)
        probs = osamp.softmax64(a, temp)
        assert abs(res.mass[b].item() - probs[s].sum()) <= 1e-6
        smallest = s[np.argmin(a[s])]
        assert abs(res.mass_without_smallest[b].item() - (probs[s].sum() - probs[smallest])) <= 1e-6


@pytest.mark.parametrize("delta", [-1, 0, 1])
def test_topp_off_by_one_matches_oracle(delta: int) -> None:
    from pck.cuda import check_topp_gpu, topp_select

    lg = logits(8, 600, seed=51)
    sel, lengths = topp_select(lg, 0.8)
    lengths = (lengths + delta).clamp(min=1)
    got = check_topp_gpu(lg, sel, lengths, 0.8, tol=0.0).passed.cpu().numpy()
    want = [osamp.check_topp(lg[b].cpu().numpy(), sel[b, : lengths[b]].cpu().numpy(), 0.8, tol=0.0) for b in range(8)]
    np.testing.assert_array_equal(got, want)
    assert got.all() == (delta == 0)


@pytest.mark.parametrize("segments", [1, 2, 7, 38, 151_936])
def test_segment_count_does_not_change_verdicts(segments: int) -> None:
    from pck.cuda import check_topk_gpu, check_topp_gpu, topk_sample, topp_select

    lg = logits(4, 151_936, seed=21, scale=2.0)
    selected = topk_sample(lg, 30)[0]
    bad = selected.clone()
    bad[1, 0] = selected[1, 1]
    ref = check_topk_gpu(lg, bad, 30, segments=1)
    got = check_topk_gpu(lg, bad, 30, segments=segments)
    assert torch.equal(got.passed, ref.passed) and ref.passed.tolist() == [True, False, True, True]
    assert torch.equal(got.min_selected, ref.min_selected) and torch.equal(got.max_rejected, ref.max_rejected)
    nucleus, lengths = topp_select(lg, 0.9)
    ref_p = check_topp_gpu(lg, nucleus, lengths, 0.9, tol=1e-5, segments=1)
    got_p = check_topp_gpu(lg, nucleus, lengths, 0.9, tol=1e-5, segments=segments)
    assert got_p.passed.all() and ref_p.passed.all()
    torch.testing.assert_close(got_p.mass, ref_p.mass, rtol=16 * 2.0**-24, atol=0)


def test_large_vocabulary_and_masked_logits() -> None:
    from pck.cuda import check_topk_gpu, check_topp_gpu, topk_sample, topp_select

    lg = logits(2, 500_000, seed=22)
    assert check_topk_gpu(lg, topk_sample(lg, 64)[0], 64).passed.all()
    nucleus, lengths = topp_select(lg, 0.5)
    assert check_topp_gpu(lg, nucleus, lengths, 0.5, tol=1e-5).passed.all()
    lg = logits(4, 1000, seed=5, scale=2.0)
    lg[:, ::7] = -math.inf
    selected, lengths = topp_select(lg, 0.9)
    res = check_topp_gpu(lg, selected, lengths, 0.9, tol=1e-5)
    assert res.passed.all() and torch.isfinite(res.mass).all()
    for b in range(4):
        assert osamp.check_topp(lg[b].cpu().numpy(), selected[b, : lengths[b]].cpu().numpy(), 0.9, tol=1e-5)


def test_rejects_bad_inputs() -> None:
    from pck.cuda import check_topk_gpu, check_topp_gpu, sharded_topk_gpu, topk_sample, topp_select

    lg = logits(2, 10, seed=0)
    sel, lengths = topp_select(lg, 0.5)
    with pytest.raises(ValueError, match="p must"):
        check_topp_gpu(lg, sel, lengths, 0.0)
    with pytest.raises(ValueError, match="tol"):
        check_topp_gpu(lg, sel, lengths, 0.5, tol=-1.0)
    with pytest.raises(RuntimeError, match="segments"):
        check_topk_gpu(lg, topk_sample(lg, 2)[0], 2, segments=11)
    with pytest.raises(RuntimeError, match="selected must be"):
        check_topk_gpu(lg, sel.int(), 1)
    with pytest.raises(ValueError, match="vocab % shards"):
        sharded_topk_gpu(lg, 2, shards=3, per_shard=1)
