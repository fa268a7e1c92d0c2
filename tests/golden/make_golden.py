"""Freezes golden vectors from the reference implementation's own Python code.

Run once in the build container, where the reference tree is mounted read-only:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference package (``<reference>/src/pck``) — never this repository's
`pck` — runs its CPU models, checkers and the GPU checker's weight-load code (which runs
on CPU tensors once `is_cuda` is satisfied), and writes the outputs next to this file.
The tests compare the oracle (and, through it, the CUDA path) against these files; they
never read the reference tree.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))  # for tests.golden.inputs

GEMV_CASES = [  # (m, n, threads): tests/gpu/test_gemv_cuda.py:122-136 plus odd shapes
    (1, 1, 32), (3, 5, 64), (7, 100, 32), (64, 1000, 32), (5, 17, 1024), (33, 4096, 128),
    (256, 4096, 256), (256, 4100, 256), (16, 14336, 512), (128, 4096, 1024), (9, 77, 64),
]  # fmt: skip
NAIVE_THREADS = [1, 2, 4, 16, 32, 256]
FP8_CASES = [(1, 1, 32), (3, 5, 64), (7, 100, 32), (5, 17, 1024), (33, 4096, 128),
             (256, 4100, 256), (64, 14336, 256)]  # fmt: skip
STORE_INPUTS_UP_TO = 70_000  # elements; larger inputs are regenerated and hash-checked


def main(reference: Path) -> None:
    sys.path.insert(0, str(reference / "src"))
    import pck  # the reference package
    from pck import checker as ref_checker
    from pck import faults as ref_faults
    from pck import fp as ref_fp
    from pck import gemv as ref_gemv
    from pck import member as ref_member
    from pck import sampling as ref_sampling
    from pck.cuda import checker as ref_gpu_checker

    from tests.golden import inputs

    assert Path(pck.__file__).resolve().is_relative_to(reference.resolve()), pck.__file__

    # -- fp constants ---------------------------------------------------------------------
    fp = {
        "tree_height": [
            [n, t, v, ref_fp.tree_height(n, t, v)]
            for n in (1, 5, 17, 100, 1000, 4096, 4100, 14336, 128256)
            for t in (1, 32, 64, 128, 256, 512, 1024)
            for v in (1, 8, 16)
        ],
        "gamma": [[k, ref_fp.gamma(k)] for k in (0, 1, 23, 63, 71, 520, 4096)],
        "gamma64": [[k, ref_fp.gamma(k, ref_fp.U64)] for k in (1, 4225, 150000)],
        "sum_up_factor": [[b, ref_fp.sum_up_factor(b)] for b in (1, 8, 64, 128, 512, 4096)],
        "softmax_eps": [[v, ref_fp.softmax_eps(v)] for v in (1, 10, 1000, 151936, 128256)],
        "softmax_eps_z": [[v, z, ref_fp.softmax_eps(v, z)] for v, z in ((1000, 4.0), (151936, 7.5))],
        "member_eps": [[v, ref_member.member_eps(v)] for v in (2, 500, 151936)],
        "member_eps32": [[v, ref_member.member_eps32(v)] for v in (2, 400, 500, 5000, 128256, 151936)],
        "bf16": [
            [float(v), float(ref_fp.bf16(np.float32(v)))]
            for v in (1.0, 1 + 2**-8, 1 + 3 * 2**-8, 1 + 2**-8 + 2**-20, -1.5, 0.0, 3.3895314e38)
        ],
        "round_up_f32": [[v, float(ref_fp.round_up_f32([v])[0])] for v in (0.0, 1.0, 0.1, 1e-40)],
    }
    # the GPU checker's host constants (src/pck/cuda/checker.py:311, 320-330)
    consts = []
    for n, block, h, checks, segs in ((4096, 128, 23, 1, 8), (4096, 64, 23, 8, None),
                                      (1000, 32, 23, 4, 1), (1000, 32, 23, 4, 1000),
                                      (14336, 128, 63, 1, None), (4100, 64, 31, 8, None),
                                      (2048, 64, 30, 8, None)):  # fmt: skip
        W = torch.zeros((block * 2, n), dtype=torch.bfloat16)
        g = torch.Generator().manual_seed(0)
        ch = _ref_gpu_checker(ref_gpu_checker, W, block, h, checks, g, segs)
        consts.append([n, block, h, checks, segs, ch.segments, ch.coef, ch.geps, ch.tau_floor])
    fp["gpu_checker_constants"] = consts
    (HERE / "fp.json").write_text(json.dumps(fp, indent=1))

    # -- GEMV models ----------------------------------------------------------------------
    out: dict[str, np.ndarray] = {}
    for m, n, t in GEMV_CASES:
        W, x = inputs.numpy_problem(m, n, seed=m * n + t)
        key = f"{m}x{n}_t{t}"
        out[f"digest_{key}"] = np.array(inputs.digest(W, x))
        if m * n <= STORE_INPUTS_UP_TO:
            out[f"W_{key}"] = inputs.bits16(W)
            out[f"x_{key}"] = inputs.bits16(x)
        out[f"coalesced_{key}"] = ref_gemv.emulate_gemv_coalesced(W, x, t).view(np.uint32)
        out[f"naive_{key}"] = ref_gemv.emulate_gemv(W, x, t).view(np.uint32)
    for t in NAIVE_THREADS:
        W, x = inputs.numpy_problem(9, 77, seed=t)
        out[f"naive_small_t{t}"] = ref_gemv.emulate_gemv(W, x, t).view(np.uint32)
    # signed zeros (tests/gpu/test_gemv_cuda.py:169-174)
    Wz, xz = np.zeros((2, 64), dtype=np.float32), -np.ones(64, dtype=np.float32)
    for t in (32, 64):
        out[f"signed_zero_coalesced_t{t}"] = ref_gemv.emulate_gemv_coalesced(Wz, xz, t).view(np.uint32)
        out[f"signed_zero_naive_t{t}"] = ref_gemv.emulate_gemv(Wz, xz, t).view(np.uint32)
    # planted shortcuts on the naive model (tests/gpu/test_checker_cuda.py:83-98)
    W, x = inputs.numpy_problem(512, 2048, seed=2)
    for name, kw in (("legit", {}), ("drop_tail4", {"drop_tail": 4}), ("acc_bf16", {"acc_bf16": True}),
                     ("partial_bf16", {"partial_bf16": True})):  # fmt: skip
        out[f"exploit_{name}"] = ref_gemv.emulate_gemv(W, x, 128, **kw).view(np.uint32)
    np.savez_compressed(HERE / "gemv.npz", **out)

    # -- FP8 --------------------------------------------------------------------------------
    out = {}
    for m, n, t in FP8_CASES:
        W, x = inputs.torch_problem(m, n, seed=m * n + t)
        Q, s = inputs.quantize_fp8_cpu(W)
        key = f"{m}x{n}_t{t}"
        out[f"digest_{key}"] = np.array(inputs.digest(Q.view(torch.uint8).numpy(), x.float().numpy()))
        out[f"Q_{key}"] = Q.view(torch.uint8).numpy() if m * n <= STORE_INPUTS_UP_TO else np.zeros(0)
        out[f"s_{key}"] = s.numpy()
        out[f"z_{key}"] = ref_gemv.emulate_gemv_coalesced(
            Q.float().numpy(), x.float().numpy(), t, vec=16
        ).view(np.uint32)
    for seed in range(6):
        Qb, xb = inputs.fp8_bit_patterns(24, 600, seed)
        out[f"patterns_z_{seed}"] = ref_gemv.emulate_gemv_coalesced(
            Qb.float().numpy(), xb.float().numpy(), 64, vec=16
        ).view(np.uint32)
        out[f"patterns_digest_{seed}"] = np.array(
            inputs.digest(Qb.view(torch.uint8).numpy(), xb.float().numpy())
        )
    np.savez_compressed(HERE / "fp8.npz", **out)

    # -- configuration 1 and the GPU checker bank -----------------------------------------
    out = {}
    g = torch.Generator().manual_seed(0)
    W = (torch.randn(4096, 4096, generator=g) * 0.02).bfloat16()
    x = torch.randn(4096, generator=g).bfloat16()
    W32, x32 = W.float().numpy(), x.float().numpy()
    out["digest"] = np.array(inputs.digest(W32, x32))
    y = ref_gemv.emulate_gemv_coalesced(W32, x32, 256)
    out["y"] = y.view(np.uint32)
    h = ref_fp.tree_height(4096, 256, 8)
    ch = _ref_gpu_checker(ref_gpu_checker, W, 128, h, 1, g, 8)
    out["r"] = ch.r.numpy()
    out["c_digest"] = np.array(inputs.digest(ch.c.numpy()))
    out["c_head"] = ch.c[:, :, :64].numpy()
    out["a_digest"] = np.array(inputs.digest(ch.a.view(torch.int16).numpy()))
    out["a_head"] = ch.a[:, :64].view(torch.int16).numpy()
    out["consts"] = np.array([ch.coef, ch.geps, ch.tau_floor, ch.segments])
    # the reference CPU checker on the honest output and on planted faults
    bank = ref_checker.WeightBank(W32, 128)
    planted = {
        "honest": y,
        "drop_tail64": ref_gemv.emulate_gemv_coalesced(
            np.where(np.arange(4096) >= 4032, 0, W32).astype(np.float32), x32, 256
        ),
        "bf16_output": ref_fp.bf16(y),
        "exponent_flip": ref_faults.flip_bit(y, 777, 27),
        "sign_flip": ref_faults.flip_bit(y, 1234, 31),
    }
    for name, yy in planted.items():
        chk = ref_checker.BlockedChecker(W32, x32, 128, h, bank)
        out[f"cpu_verdict_{name}"] = chk.verdict(yy, np.random.default_rng(7), checks=4)
        out[f"planted_digest_{name}"] = np.array(inputs.digest(yy))
    np.savez_compressed(HERE / "config1.npz", **out)

    # -- a small bank stored whole -------------------------------------------------------
    out = {}
    Wn, xn = inputs.numpy_problem(256, 1000, seed=1)
    Wt = torch.from_numpy(Wn).bfloat16()
    g = torch.Generator().manual_seed(1)
    ch = _ref_gpu_checker(ref_gpu_checker, Wt, 32, 23, 4, g, 3)
    out["r"], out["c"] = ch.r.numpy(), ch.c.numpy()
    out["a"] = ch.a.view(torch.int16).numpy()
    out["consts"] = np.array([ch.coef, ch.geps, ch.tau_floor, ch.segments])
    out["digest"] = np.array(inputs.digest(Wn, xn))
    np.savez_compressed(HERE / "bank_small.npz", **out)

    # round_up_bf16 known answers (tests/gpu/test_round_up_bf16.py:20-38)
    vals = torch.tensor([0.0, 1.0, 1 + 2**-30, 1 + 2**-8, 3.0, 0.1, 1e-30, 3.3e38, 3.4e38],
                        dtype=torch.float64)  # fmt: skip
    rb = ref_gpu_checker.round_up_bf16(vals)
    (HERE / "round_up_bf16.json").write_text(
        json.dumps({"in": vals.tolist(), "out": [float(v) for v in rb.float()]})
    )

    # -- membership ------------------------------------------------------------------------
    out = {}
    logits, tokens, top_k, top_p, greedy = inputs.member_case_ties()
    r = ref_member.check_members(torch.tensor(logits), torch.tensor(tokens), torch.tensor(top_k),
                                 torch.tensor(top_p), torch.tensor(greedy))  # fmt: skip
    _store_members(out, "ties", r, logits, tokens, top_k, top_p, greedy, ref_member)
    logits, tokens, top_k, top_p = inputs.member_case_kth_ties()
    r = ref_member.check_members(torch.tensor(logits), torch.tensor(tokens),
                                 torch.tensor(top_k, dtype=torch.int32), torch.tensor(top_p))  # fmt: skip
    _store_members(out, "kth_ties", r, logits, tokens, top_k, top_p, None, ref_member)
    logits, tokens = inputs.member_case_wide()
    tp = np.full(16, 0.99)
    r = ref_member.check_members(torch.tensor(logits), torch.tensor(tokens),
                                 top_p=torch.tensor(tp, dtype=torch.float64))  # fmt: skip
    _store_members(out, "wide", r, logits, tokens, None, tp, None, ref_member)
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((4, 50)).astype(np.float32)
    tokens = np.array([-1, 50, 10_000, int(logits[3].argmax())])
    tk = np.array([5, 5, 5, 20])
    r = ref_member.check_members(torch.tensor(logits), torch.tensor(tokens),
                                 torch.tensor(tk, dtype=torch.int32),
                                 torch.full((4,), 0.9, dtype=torch.float64),
                                 top_k_host=np.array([5, 5, 5, 5]))  # fmt: skip
    out["bad_ids_ok"] = r["ok"].numpy()
    out["bad_ids_above"] = r["above"].numpy()
    lg, tok, tk, tp, faulty = inputs.member_case_lm_head(64, 128256, seed=5)
    r = ref_member.check_members(lg, tok, tk, tp)
    out["lm_head_ok"], out["lm_head_above"] = r["ok"].numpy(), r["above"].numpy()
    out["lm_head_mass"], out["lm_head_faulty"] = r["mass_above"].numpy(), faulty.numpy()
    out["lm_head_digest"] = np.array(inputs.digest(lg.numpy(), tok.numpy()))
    np.savez_compressed(HERE / "member.npz", **out)

    # -- sampling set checks ---------------------------------------------------------------
    out = {}
    for seed in range(5):
        rows, vocab, k = 8, 2000, 20
        lg = inputs.sampling_logits(rows, vocab, seed, ties=True)
        sel = np.stack([ref_sampling.topk_reference(lg[b], k) for b in range(rows)])
        rng = np.random.default_rng(seed)
        for b in range(rows):
            rejected = np.setdiff1d(np.arange(vocab), sel[b])
            sel[b, rng.integers(k)] = int(rng.choice(rejected))
        out[f"swap_sel_{seed}"] = sel
        out[f"swap_verdict_{seed}"] = np.array(
            [ref_sampling.check_topk(lg[b], sel[b], k) for b in range(rows)]
        )
    lg = inputs.sampling_logits(8, 500, 11)
    for delta in (-1, 0, 1):
        verdicts, sels = [], []
        for b in range(8):
            nuc = ref_sampling.topp_reference(lg[b], 0.8)
            length = min(max(nuc.size + delta, 1), 500)
            order = np.lexsort((np.arange(500), -lg[b].astype(np.float64)))
            sel = order[:length]
            sels.append(np.pad(sel, (0, 500 - length), constant_values=-1))
            verdicts.append(ref_sampling.check_topp(lg[b], sel, 0.8, tol=0.0))
        out[f"topp_delta{delta}_sel"] = np.stack(sels)
        out[f"topp_delta{delta}_verdict"] = np.array(verdicts)
    lg = inputs.sampling_logits(8, 4096, 3)
    lg[0, :16] = 100.0 + np.arange(16, dtype=np.float32)
    for per_shard in (4, 16):
        sel = np.stack([ref_faults.sharded_topk(lg[b], 16, 8, per_shard) for b in range(8)])
        out[f"sharded_{per_shard}_sel"] = sel
        out[f"sharded_{per_shard}_verdict"] = np.array(
            [ref_sampling.check_topk(lg[b], sel[b], 16) for b in range(8)]
        )
    np.savez_compressed(HERE / "sampling.npz", **out)
    print("golden fixtures written to", HERE)


def _ref_gpu_checker(mod, W, block, height, checks, generator, segments):
    """Runs the reference GpuBlockedChecker's weight-load code on a CPU tensor."""

    class CpuAsCuda(torch.Tensor):
        @property
        def is_cuda(self) -> bool:  # only the constructor's device check reads this
            return True

    # the default segment count reads the SM count: answer with a B200's 148
    from types import SimpleNamespace
    from unittest import mock

    props = SimpleNamespace(multi_processor_count=B200_SMS)
    with mock.patch.object(torch.cuda, "get_device_properties", lambda *_: props):
        return mod.GpuBlockedChecker(W.as_subclass(CpuAsCuda), block, height, checks=checks,
                                     generator=generator, segments=segments)  # fmt: skip


B200_SMS = 148


def _store_members(out, name, r, logits, tokens, top_k, top_p, greedy, ref_member) -> None:
    out[f"{name}_ok"] = r["ok"].numpy()
    out[f"{name}_above"] = r["above"].numpy()
    out[f"{name}_mass"] = r["mass_above"].numpy()
    rows = logits.shape[0]
    ref_ok, ref_above, ref_mass = [], [], []
    vocab = logits.shape[1]
    for i in range(rows):
        k = None if top_k is None or top_k[i] >= vocab else int(top_k[i])
        p = None if top_p is None or top_p[i] >= 1.0 else float(top_p[i])
        g = bool(greedy[i]) if greedy is not None else False
        v = ref_member.check_member(logits[i], int(tokens[i]), k, p, greedy=g)
        ref_ok.append(v.ok)
        ref_above.append(v.above)
        ref_mass.append(v.mass_above)
    out[f"{name}_member_ok"] = np.array(ref_ok)
    out[f"{name}_member_above"] = np.array(ref_above)
    out[f"{name}_member_mass"] = np.array(ref_mass)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(Path(sys.argv[1]))
