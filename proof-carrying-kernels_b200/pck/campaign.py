"""Fault-injection campaign of the blocked checker on the GPU (the B200 counterpart of the
reference's harness/campaign.py).

On a 4096 x 4096 bfloat16 GEMV with seeded inputs (Gaussian, Student-t, mixed-scale and
LLM-like outlier activations in turn):

- honest runs: both bit-exact GEMV kernels (coalesced and naive tree), every output block
  checked with K sign draws; a false alarm is a failed (check, block) pair, and the
  largest |rho| / tau shows how close a legitimate output came to the threshold;
- planted shortcuts, computed by untrusted torch code on the GPU in the reference's exploit
  semantics (src/pck/gemv.py:14-57): the last 64 columns dropped (naive tree; for the
  coalesced tree the columns >= n - 64 zeroed), bfloat16 running accumulators, bfloat16
  per-thread partial sums, a bfloat16-rounded output, and exponent or sign bit flips at a
  rate of 1e-4 per output element. A block is faulty if its output differs from the honest
  one; it is caught if any of its K checks fails. For a block with a single wrong element
  the checker guarantees detection once that error exceeds 2 tau (for every sign draw);
  errors spread over many elements of a block (e.g. a rounded output) can cancel in r . y,
  so for them, and below 2 tau, detection is reported as a rate.

    python -m pck.campaign [--inputs N] [--batch B] [--checks K] [--seed S]

With ``--kernel tc`` the honest outputs come from the tensor-core GEMV (`gemv_tc`, decode
batches of up to 256 columns), whose summation order is the tensor core's: its checker
takes the declared height `tc_height(n)`, which rests on a hypothesis about the MMA's
internal rounding (at most 8 unit roundoffs per step). The campaign then counts false alarms
of the checks fused into the GEMV call, reports the largest |rho| / tau and the largest
observed error as a fraction of the declared bound gamma_h sum |w||x| (binary64 reference),
and plants bf16-rounded outputs and bit flips on the tensor-core outputs.

Prints one JSON object with the counts.
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from pck.cuda import GpuBlockedChecker, gemv_coalesced, gemv_naive, gemv_tc, tc_height
from pck.fp import U32, gamma, tree_height

N = 4096
THREADS = 256
DISTS = ("gauss", "student-t", "mixed-scale", "outliers")


def activations(kind: str, batch: int, n: int, gen: torch.Generator) -> torch.Tensor:
    """A batch of seeded activation rows of one distribution (bfloat16, on the CPU)."""
    if kind == "gauss":
        x = torch.randn(batch, n, generator=gen)
    elif kind == "student-t":  # 3 degrees of freedom: normal / sqrt(chi2_3 / 3)
        z = torch.randn(batch, n, generator=gen)
        chi = torch.randn(batch, n, 3, generator=gen).square().sum(-1) / 3.0
        x = z / chi.sqrt()
    elif kind == "mixed-scale":
        x = torch.randn(batch, n, generator=gen) * torch.exp2(torch.randint(-20, 21, (batch, n), generator=gen).float())
    elif kind == "outliers":
        x = torch.randn(batch, n, generator=gen)
        for b in range(batch):
            x[b, torch.randperm(n, generator=gen)[: n // 100]] *= 100.0
    else:
        raise ValueError(kind)
    return x.bfloat16()


def _bf16(v: torch.Tensor) -> torch.Tensor:
    return v.bfloat16().float()


def naive_shortcut(W: torch.Tensor, X: torch.Tensor, *, acc_bf16: bool = False, partial_bf16: bool = False,
                   drop_tail: int = 0) -> torch.Tensor:  # fmt: skip
    """The naive tree (thread t sums a contiguous chunk, then adjacent pairs) with the
    reference's exploits, in binary32 on the GPU: untrusted code under test."""
    m, n = W.shape
    chunk = -(-n // THREADS)
    P = W.float()[None] * X.float()[:, None, :]  # exact products, (batch, m, n)
    if drop_tail:
        P[:, :, n - drop_tail :] = 0
    P = torch.nn.functional.pad(P, (0, chunk * THREADS - n)).view(X.size(0), m, THREADS, chunk)
    acc = P[..., 0].clone()
    for j in range(1, chunk):
        acc = acc + P[..., j]
        if acc_bf16:
            acc = _bf16(acc)
    if partial_bf16:
        acc = _bf16(acc)
    while acc.size(-1) > 1:
        acc = acc[..., 0::2] + acc[..., 1::2]
    return acc[..., 0].contiguous()


def flip_bits(Y: torch.Tensor, rate: float, gen: torch.Generator) -> torch.Tensor:
    """Exponent (bits 23-30) or sign (bit 31) flips at ``rate`` per element."""
    hit = torch.rand(Y.shape, generator=gen) < rate
    bit = torch.randint(23, 32, Y.shape, generator=gen)
    mask = torch.where(hit, torch.ones_like(bit) << bit, torch.zeros_like(bit)).to(torch.int32)
    return (Y.view(torch.int32) ^ mask.to(Y.device)).view(torch.float32)


class Tally:
    def __init__(self) -> None:
        self.faulty = self.caught = self.single = self.single_caught = 0

    def add(self, honest: torch.Tensor, bad: torch.Tensor, verdict: torch.Tensor, tau: torch.Tensor,
            block: int) -> None:  # fmt: skip
        b, m = honest.shape
        diff = (bad.double() - honest.double()).abs().view(b, m // block, block)
        diff = torch.where(torch.isnan(diff), torch.full_like(diff, float("inf")), diff)
        wrong = (diff > 0).sum(dim=2)
        delta = diff.amax(dim=2)
        faulty = wrong > 0
        caught = ~verdict
        single = (wrong == 1) & (delta > 2 * tau.amax(dim=1))  # the guaranteed case
        self.faulty += int(faulty.sum())
        self.caught += int((faulty & caught).sum())
        self.single += int(single.sum())
        self.single_caught += int((single & caught).sum())

    def as_dict(self) -> dict:
        return {"faulty_blocks": self.faulty, "caught": self.caught,
                "rate": self.caught / self.faulty if self.faulty else None,
                "single_element_above_2tau": self.single,
                "single_element_above_2tau_caught": self.single_caught}  # fmt: skip


def run(inputs: int, batch: int, checks: int, block: int, seed: int, device: torch.device) -> dict:
    gen = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, N, generator=gen) * 0.02).bfloat16().to(device)
    coal = GpuBlockedChecker(W, block, tree_height(N, THREADS, 8), checks=checks, generator=gen)
    naive = GpuBlockedChecker(W, block, tree_height(N, THREADS, 1), checks=checks, generator=gen)
    alarms = {"coalesced": 0, "naive": 0}
    block_checks = {"coalesced": 0, "naive": 0}
    worst = {"coalesced": 0.0, "naive": 0.0}
    tallies = {k: Tally() for k in ("drop_tail", "acc_bf16", "partial_bf16", "bf16_output", "bit_flips")}
    flips = torch.Generator().manual_seed(seed + 1)
    start = time.perf_counter()
    done = 0
    while done < inputs:
        b = min(batch, inputs - done)
        X = activations(DISTS[(done // batch) % len(DISTS)], b, N, gen).to(device)
        honest_c = gemv_coalesced(W, X, THREADS)
        honest_n = torch.stack([gemv_naive(W, X[i], THREADS) for i in range(b)])
        for name, Y, ch in (("coalesced", honest_c, coal), ("naive", honest_n, naive)):
            res = ch.check(X, Y)
            alarms[name] += int((~res.passed).sum())
            block_checks[name] += res.passed.numel()
            worst[name] = max(worst[name], float((res.rho.abs() / res.tau).max()))
        tau_n = naive.check(X, honest_n).tau
        tau_c = coal.check(X, honest_c).tau
        Xt = X.clone()
        Xt[:, N - 64 :] = 0
        for name, bad, ch, honest, tau in (
            ("drop_tail", naive_shortcut(W, X, drop_tail=64), naive, honest_n, tau_n),
            ("acc_bf16", naive_shortcut(W, X, acc_bf16=True), naive, honest_n, tau_n),
            ("partial_bf16", naive_shortcut(W, X, partial_bf16=True), naive, honest_n, tau_n),
            ("bf16_output", _bf16(honest_c), coal, honest_c, tau_c),
            ("bit_flips", flip_bits(honest_c, 1e-4, flips), coal, honest_c, tau_c),
        ):
            tallies[name].add(honest, bad, ch.check(X, bad.contiguous()).verdict, tau, block)
        # the coalesced tree with its tail columns zeroed, checked against the true x
        bad = gemv_coalesced(W, Xt, THREADS)
        tallies["drop_tail"].add(honest_c, bad, coal.check(X, bad).verdict, tau_c, block)
        done += b
    torch.cuda.synchronize()
    return {
        "config": {"W": [N, N], "inputs": inputs, "batch": batch, "checks": checks, "block": block, "seed": seed,
                   "distributions": list(DISTS)},
        "honest": {"block_checks": block_checks, "false_alarms": alarms, "max_rho_over_tau": worst},
        "planted": {k: t.as_dict() for k, t in tallies.items()},
        "seconds": round(time.perf_counter() - start, 1),
    }  # fmt: skip


def run_tc(inputs: int, batch: int, checks: int, block: int, seed: int, device: torch.device,
           bound_every: int = 8) -> dict:  # fmt: skip
    """The campaign on the tensor-core GEMV: honest batches checked by the call's own fused
    check (the production path), every ``bound_every``-th batch also measured against the
    declared bound in binary64, and the output faults planted on its outputs."""
    gen = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, N, generator=gen) * 0.02).bfloat16().to(device)
    height = tc_height(N)
    checker = GpuBlockedChecker(W, block, height, checks=checks, generator=gen)
    W64 = W.double()
    g = gamma(height, U32)
    alarms = block_checks = 0
    worst_ratio = worst_bound = 0.0
    per_dist = {d: {"block_checks": 0, "false_alarms": 0, "max_rho_over_tau": 0.0} for d in DISTS}
    tallies = {k: Tally() for k in ("bf16_output", "bit_flips")}
    flips = torch.Generator().manual_seed(seed + 1)
    start = time.perf_counter()
    done = calls = 0
    while done < inputs:
        b = min(batch, inputs - done)
        dist = DISTS[calls % len(DISTS)]
        X = activations(dist, b, N, gen).to(device)
        Y, res = gemv_tc(W, X, checker)
        fa = int((~res.passed).sum())
        ratio = float((res.rho.abs() / res.tau).max())
        alarms += fa
        block_checks += res.passed.numel()
        worst_ratio = max(worst_ratio, ratio)
        d = per_dist[dist]
        d["block_checks"] += res.passed.numel()
        d["false_alarms"] += fa
        d["max_rho_over_tau"] = max(d["max_rho_over_tau"], ratio)
        if calls % bound_every == 0:
            X64 = X.double()
            err = (Y.double() - X64 @ W64.T).abs()
            mag = X64.abs() @ W64.abs().T
            worst_bound = max(worst_bound, float((err / (g * mag).clamp(min=1e-300)).max()))
            # planted output faults, checked by the standalone check (16 columns a call)
            bad_r = _bf16(Y)
            bad_f = flip_bits(Y, 1e-4, flips)
            for b0 in range(0, b, 16):
                b1 = min(b, b0 + 16)
                Xs = X[b0:b1].contiguous()
                tau = res.tau[b0:b1]
                for name, bad in (("bf16_output", bad_r), ("bit_flips", bad_f)):
                    v = checker.check(Xs, bad[b0:b1].contiguous()).verdict
                    tallies[name].add(Y[b0:b1], bad[b0:b1], v, tau, block)
        done += b
        calls += 1
    torch.cuda.synchronize()
    return {
        "config": {"kernel": "tcgen05 gemv_tc (fused check)", "W": [N, N], "inputs": inputs, "batch": batch,
                   "checks": checks, "block": block, "seed": seed, "height": height, "distributions": list(DISTS)},
        "honest": {"block_checks": block_checks, "false_alarms": alarms, "max_rho_over_tau": worst_ratio,
                   "max_error_over_declared_bound": worst_bound, "bound_sampled_every": bound_every,
                   "per_distribution": per_dist},
        "planted": {k: t.as_dict() for k, t in tallies.items()},
        "seconds": round(time.perf_counter() - start, 1),
    }  # fmt: skip


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--kernel", choices=["tree", "tc"], default="tree",
                   help="tree: the bit-exact coalesced and naive trees; tc: the tensor-core GEMV")
    p.add_argument("--inputs", type=int, default=100_000)
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--checks", type=int, default=8)
    p.add_argument("--block", type=int, default=128)
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args()
    fn = run_tc if a.kernel == "tc" else run
    print(json.dumps(fn(a.inputs, a.batch, a.checks, a.block, a.seed, torch.device("cuda", 0))), flush=True)


if __name__ == "__main__":
    main()
