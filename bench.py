"""Checked decode-layer benchmark (the driver's contract: one JSON line from rank 0).

Workload: the Llama-3-8B decode-layer GEMV set (q 4096x4096, k/v 1024x4096, o 4096x4096,
gate/up 14336x4096, down 4096x14336), bfloat16 weights ~N(0, 0.02^2), activations ~N(0, 1)
with 1% outlier channels x20, every output checked by the trusted blocked checker
(b = 128, K = 1). A step is one decode layer: four launches of the persistent streaming
kernel (q/k/v share their input, o, gate/up share theirs, down), each with its checks'
bank rows fused into the same pass over memory. The block verdicts are decided inside the
next streaming launch (`pck_gemv_pipelined`: o's launch decides q/k/v's blocks, ..., the next
layer's q/k/v launch decides down's), so a step still decides all seven checks, with no
launch of its own; `--verdicts launch` instead ends the step with one verdict-kernel launch
for all seven (the reference runs one checker launch per layer). Captured in a CUDA graph.
With N GPUs every matrix is row-sharded by whole checker blocks and one all-gather per
step assembles the outputs and verdict bits: by default this library's peer-memory kernel
(each rank stores its slice into every peer over NVLink), `--gather nccl` for NCCL's.

metric: checked-GEMV HBM throughput = algorithmic bytes of the step (weights, activations,
outputs, checksum bank, verdicts) / device time, GB/s, over all ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "proof-carrying-kernels_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "checked GEMV HBM GB/s (Llama-3-8B decode layer, b=128 blocks, K=1)"
UNIT = "GB/s"
VERDICTS = {
    "carried": "decided inside the next streaming launch (pck_gemv_pipelined); the next layer's first launch "
               "decides down's blocks",
    "launch": "one verdict-kernel launch per layer after the four GEMV launches",
}  # fmt: skip
SCOPE = {"carried": "4 stream_kernel launches, each deciding the previous launch's checks",
         "launch": "4 stream_kernel launches + 1 verdict_kernel launch"}  # fmt: skip
L2_BYTES = 126 * 2**20
LLAMA3_GROUP_NAMES = [["q", "k", "v"], ["o"], ["gate", "up"], ["down"]]


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def profile_traffic(weights: str = "bf16") -> float | None:
    """DRAM bytes per step (the four streaming launches) from the committed ncu summary of
    the same weight format."""
    name = "stream_kernel_decode_layer.md" if weights == "bf16" else f"stream_kernel_decode_layer_{weights}.md"
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_step:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")  # fmt: skip

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"pck_clocks_{os.getpid()}.csv"

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)],
                stdout=self.path.open("w"), stderr=subprocess.DEVNULL,
            )  # fmt: skip
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}  # fmt: skip


def outlier_x(n: int, batch: int, gen: torch.Generator) -> torch.Tensor:
    x = torch.randn(batch, n, generator=gen)
    for b in range(batch):
        idx = torch.randperm(n, generator=gen)[: max(1, n // 100)]
        x[b, idx] *= 20.0
    return x.bfloat16()


def build_layer(args, rank: int, world: int, device: torch.device, keep_full: bool = False, share=None):
    """Sharded weights, inputs, checkers and the launch objects of one decode layer. With
    ``keep_full``, also the unsharded weights of every projection (for the check that the
    gathered outputs equal the single-GPU ones). With ``share`` (a layer built before), a
    further copy of the layer in memory of its own (the same values) that writes the same
    output, verdict and exchange buffers and reads the same activations, as the layers of a
    model do."""
    from pck.cuda import GpuBlockedChecker
    from pck.cuda.plan import LLAMA3_8B_GROUPS, GemvLaunch, VerdictLaunch
    from pck.cuda.sharded import Exchange, shard_rows
    from pck.fp import tree_height

    if share is None:
        names = [p for g in LLAMA3_8B_GROUPS for p in g]
        ms = [m for _, m, _ in names]
        # one all-gather per step moves the outputs and the verdict bits of every projection
        ex = Exchange([(ms, args.block, args.batch, torch.float32),
                       ([m // args.block for m in ms], 1, args.checks, torch.bool)], world, rank, device)  # fmt: skip
        ex_plain = Exchange([(ms, args.block, args.batch, torch.float32)], world, rank, device)
        gen = torch.Generator().manual_seed(0)
        # the layer's activations in one device buffer (each group's x a 16-byte aligned view),
        # so a step's inputs arrive with one host-to-device copy
        host_x = [outlier_x(group[0][2], args.batch, gen) for group in LLAMA3_8B_GROUPS]
        x_all = torch.cat([h.reshape(-1) for h in host_x]).to(device)
        views, off = [], 0
        for h in host_x:
            views.append(x_all[off : off + h.numel()].view(h.shape if args.batch > 1 else h.shape[1:]))
            off += h.numel()
    else:
        ex, ex_plain, x_all, views = share
    ys, vs = ex.parts
    groups, plain, xs, full, j = [], [], [], [], 0
    for gi, group in enumerate(LLAMA3_8B_GROUPS):
        x = views[gi]
        xs.append(x)
        items, items_plain, y_views, p_views, y_plain = [], [], [], [], []
        for _name, m, nn in group:
            shard = shard_rows(m, args.block, world, rank)
            dgen = torch.Generator(device=device).manual_seed(1000 + j)
            W_all = (torch.randn(m, nn, generator=dgen, device=device) * 0.02).bfloat16()
            W = W_all[shard.row0 : shard.row1].contiguous()
            vec = 8
            if args.weights == "e4m3":  # config 3: per-row E4M3 quantisation, checked against Q
                from pck.cuda import quantize_fp8

                W, vec = quantize_fp8(W)[0], 16
                if keep_full:
                    W_all = quantize_fp8(W_all)[0]
            full.append(W_all if keep_full else None)
            del W_all
            checker = GpuBlockedChecker(W.to(torch.bfloat16), args.block, tree_height(nn, args.threads, vec),
                                        checks=args.checks, generator=torch.Generator().manual_seed(2000 + j))  # fmt: skip
            items.append((W, x, checker))
            items_plain.append((W, x, None))
            y_views.append(ys.local_view(j))
            p_views.append(vs.local_view(j))
            y_plain.append(ex_plain.parts[0].local_view(j))
            j += 1
        groups.append(GemvLaunch(items, args.threads, ys=y_views, passed=p_views, verdicts=False))
        plain.append(GemvLaunch(items_plain, args.threads, ys=y_plain))
    verdict = VerdictLaunch(groups)
    if not getattr(args, "no_prefetch", False):  # unchecked launches prefetch the next one's first pieces too
        for i, g in enumerate(plain):
            g.verdicts = False
            g.set_next(plain[(i + 1) % len(plain)])
    torch.cuda.synchronize()
    build_layer.x_all = x_all  # the buffer behind xs (one copy per step in the end-to-end reading)
    build_layer.share = (ex, ex_plain, x_all, views)
    return groups, verdict, plain, xs, ex, ex_plain, full


def layer_copies(layer_bytes: int, steps: int) -> int:
    """Copies of the layer a rank rotates through, one per step, so that the weights it reads
    between two uses of the same bytes exceed L2 by half (a row shard at 4 or 8 GPUs fits in
    L2 alone). The smallest count at least that for which some divisor of ``steps`` up to
    GRAPH_STEPS is a multiple of it (the graphs then replay whole rotations)."""
    need = max(1, -(-int(1.5 * L2_BYTES) // max(1, layer_bytes)))
    for copies in range(need, GRAPH_STEPS + 1):
        if any(steps % d == 0 and d % copies == 0 for d in range(copies, min(steps, GRAPH_STEPS) + 1)):
            return copies
    return max(1, graph_steps(steps))


def rotation(fns):
    """One call runs the next of ``fns`` in turn (a step of the next layer copy)."""
    state = {"next": 0}

    def step() -> None:
        fns[state["next"] % len(fns)]()
        state["next"] += 1

    return step


# Consecutive layer steps captured in one CUDA graph at most: a decode graph holds every
# layer of the model (Llama-3-8B has 32), so only one step in that many pays the graph
# launch boundary.
GRAPH_STEPS = 32


def graph_steps(steps: int, copies: int = 1) -> int:
    """Steps per captured graph: the largest divisor of ``steps`` up to GRAPH_STEPS (a multiple
    of ``copies`` where one exists), so the timed region replays whole graphs and holds exactly
    ``steps`` steps."""
    ds = [d for d in range(1, min(steps, GRAPH_STEPS) + 1) if steps % d == 0]
    whole = [d for d in ds if d % copies == 0]
    return max(whole or ds)


def cuda_graph(fn, steps: int = 1) -> tuple[torch.cuda.CUDAGraph, int]:
    """A graph of ``steps`` consecutive calls of ``fn`` (run once eagerly first)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(steps):
            fn()
    torch.cuda.synchronize()
    return g, steps


def timed(graph: tuple[torch.cuda.CUDAGraph, int], steps: int, warmup: int, world: int) -> float:
    """Seconds per step: max over ranks of the CUDA-event time of exactly ``steps`` steps
    (``steps`` a multiple of the graph's steps), after at least ``warmup`` steps."""
    g, per = graph
    if steps % per:
        raise ValueError(f"steps ({steps}) must be a multiple of the graph's {per} steps")
    for _ in range(-(-warmup // per)):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps // per):
        g.replay()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms / 1e3 / steps


def e2e_step_time(layers, x_all, ex, steps: int, warmup: int, world: int) -> tuple[float, int, int]:
    """The public API with host buffers (`pck.cuda.plan.CapturedStep`): every step copies the
    layer's activations from pinned host memory, runs the launches of the next layer copy in
    ``layers`` (and the gather), and copies every output and verdict bit back to pinned host
    memory; one graph launch per step. Device time per step, max over ranks."""
    from pck.cuda.plan import CapturedStep

    hx = [x_all.cpu().pin_memory()]  # x_all: the buffer the layer's activations are views of
    hout = torch.empty(ex.gathered.shape, dtype=ex.gathered.dtype, pin_memory=True)

    def body_of(launches):
        def body() -> None:
            for g in launches:
                g.launch()
            if world > 1:
                ex.gather()

        return body

    result = ex.gathered if world > 1 else ex.local
    hres = hout if world > 1 else torch.empty(ex.local.shape, dtype=ex.local.dtype, pin_memory=True)
    captured = [CapturedStep(body_of(launches), [(hx[0], x_all)], [(result, hres)]) for launches in layers]
    step = rotation([c.run for c in captured])
    for _ in range(-(-warmup // len(captured)) * len(captured)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    h2d, d2h = captured[0].h2d_bytes, captured[0].d2h_bytes
    del step, captured
    return ms / 1e3 / steps, h2d, d2h


def launch_times(fn_sets, steps: int, world: int) -> list[float]:
    """Device time of each launch of a step, in ms: the step (the launches of the next layer
    copy in ``fn_sets``) issued eagerly ``steps`` times with a CUDA event between consecutive
    launches (on the launching stream), averaged. The events keep each launch from overlapping
    its neighbour, so the sum is a little above the graph's time per step."""
    nf = len(fn_sets[0])
    events = [torch.cuda.Event(enable_timing=True) for _ in range(nf + 1)]
    totals = [0.0] * nf
    for s in range(3 * len(fn_sets)):
        for f in fn_sets[s % len(fn_sets)]:
            f()
    torch.cuda.synchronize()
    for s in range(steps):
        fns = fn_sets[s % len(fn_sets)]
        events[0].record()
        for i, f in enumerate(fns):
            f()
            events[i + 1].record()
        torch.cuda.synchronize()
        for i in range(len(fns)):
            totals[i] += events[i].elapsed_time(events[i + 1])
    out = [t / steps for t in totals]
    if world > 1:
        t = torch.tensor(out, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        out = t.tolist()
    return [round(v, 5) for v in out]


def all_ranks(flag: bool, world: int) -> bool:
    """True iff ``flag`` holds on every rank."""
    if world == 1:
        return flag
    t = torch.tensor([1 if flag else 0], device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
    return bool(t.item())


def gathered_layer_matches(groups, xs, ex, full, world: int, rank: int) -> bool | None:
    """Multi-GPU correctness of the timed path, after a step has run: every rank's copy of
    the gathered verdict bits passes every block, and on rank 0 every projection's gathered
    output equals, bit for bit, the output of the unsharded matrix (the single-GPU result).
    The same answer on every rank. None at one GPU."""
    from pck.cuda import gemv_coalesced, gemv_fp8

    if world == 1:
        return None
    ys, vs = ex.parts
    ok = all(bool(vs.assemble(j).all()) for j in range(len(vs.ms)))
    if rank == 0:
        j = 0
        for g, x in zip(groups, xs, strict=True):
            for _ in g.items:
                W = full[j]
                y = gemv_fp8(W, x) if W.dtype == torch.float8_e4m3fn else gemv_coalesced(W, x)
                ok = ok and torch.equal(ys.assemble(j).view(torch.int32), y.view(torch.int32))
                j += 1
    return all_ranks(ok, world)


LM_VOCAB, LM_N, LM_BATCH = 128256, 4096, 64


def lm_head_reading(rank: int, world: int, device, steps: int, warmup: int, gather: str = "peer") -> dict:
    """Config 5: the Llama-3 LM head W (128256, 4096) bfloat16 at decode batch 64, row-sharded
    by whole 128-row blocks over the ranks, each rank's slice checked in the same call as its
    tensor-core GEMV; one all-gather of logits and verdict bits; top-k 50 / top-p 0.9 sampling
    at temperature 1 (untrusted torch) with 1% of the tokens replaced by the row's lowest
    logit; the fused membership check of every token. Activations are scaled so that the
    logits are ~N(0, 3^2). Device times of CUDA graphs, max over ranks."""
    from pck.cuda import gemv_tc
    from pck.cuda.lm_head import CheckedLMHead, TopKTopPSampler, membership
    from pck.cuda.sharded import shard_rows

    sh = shard_rows(LM_VOCAB, 128, world, rank)
    gen = torch.Generator(device=device).manual_seed(5000)
    W_all = (torch.randn(LM_VOCAB, LM_N, generator=gen, device=device) * 0.02).bfloat16()
    X = (torch.randn(LM_BATCH, LM_N, generator=gen, device=device) * (3.0 / (0.02 * LM_N**0.5))).bfloat16()
    W = W_all[sh.row0 : sh.row1].contiguous()
    if not (world > 1 and rank == 0):
        del W_all
        W_all = None
    head = CheckedLMHead(W, X, LM_VOCAB, world=world, rank=rank, generator=torch.Generator().manual_seed(5001))
    if world > 1 and gather == "peer":
        head.exchange.use_peer_memory()
    torch.manual_seed(5002)  # the sampler's draws: the same on every rank
    sampler = TopKTopPSampler(LM_BATCH, LM_VOCAB, k=50, p=0.9, temperature=1.0, device=device, fault_rate=0.01)
    counts = torch.zeros(4, dtype=torch.int64, device=device)  # steps all passed, planted, caught, false alarms

    def sample_and_check() -> None:
        sampler(head.logits)
        ok = membership(head.logits, sampler)["ok"]
        inj = sampler.injected
        counts.add_(torch.stack([head.passed.all().to(torch.int64), inj.sum(), (inj & ~ok).sum(), (~inj & ~ok).sum()]))

    def full_step() -> None:
        head.forward()
        sample_and_check()

    per = graph_steps(steps)
    g_gemv = cuda_graph(head.gemv.launch, per)
    g_forward = cuda_graph(head.forward, per)
    sampler(head.logits)
    g_member = cuda_graph(lambda: membership(head.logits, sampler), per)
    g_full = cuda_graph(full_step, per)
    counts.zero_()
    torch.cuda.synchronize()
    t_gemv = timed(g_gemv, steps, warmup, world)
    t_forward = timed(g_forward, steps, warmup, world)
    t_member = timed(g_member, steps, warmup, world)
    counts.zero_()
    t_full = timed(g_full, steps, warmup, world)
    torch.cuda.synchronize()
    replays = (-(-warmup // per) + steps // per) * per  # steps the counters saw
    passed_steps, planted, caught, false_alarms = (int(v) for v in counts.tolist())
    matches = None
    if world > 1:  # rank 0: the gathered logits against the unsharded GEMV, bit for bit
        ok = True
        if rank == 0:
            ok = torch.equal(gemv_tc(W_all, X, full_k=True).view(torch.int32), head.logits.view(torch.int32))
        matches = all_ranks(ok, world)
    local_bytes = head.gemv_bytes
    total = torch.tensor([float(local_bytes)], device=device)
    if world > 1:
        torch.distributed.all_reduce(total)
    gemv_gbs = float(total.item()) / t_gemv / 1e9
    peak = float(measured_peaks()["hbm_gbs"])
    del g_gemv, g_forward, g_member, g_full
    if world > 1:
        head.exchange.close()
    return {
        "workload": "Llama-3 LM head 128256x4096 bf16, batch 64, row-sharded checked tcgen05 GEMV + all-gather "
                    "+ top-k 50 / top-p 0.9 sampling + fused membership check (1% planted non-members)",
        "parallelism": f"row-shard x{world}" if world > 1 else "single",
        "gather": gather if world > 1 else None,
        "ms_per_step": round(t_full * 1e3, 4), "tokens_per_s": round(LM_BATCH / t_full),
        "gemv_ms": round(t_gemv * 1e3, 4), "gemv_and_gather_ms": round(t_forward * 1e3, 4),
        "gather_ms": round((t_forward - t_gemv) * 1e3, 4) if world > 1 else 0.0,
        "membership_ms": round(t_member * 1e3, 4),
        "gemv_GB_per_s": round(gemv_gbs, 1),
        "roofline": {"bound": "hbm", "achieved": round(gemv_gbs / world, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gemv_gbs / world / peak, 4),
                     "scope": "per GPU: the checked GEMV launch (W slice, X, logits, bank, verdicts)"},
        "all_blocks_passed": passed_steps == replays, "planted": planted, "caught": caught,
        "false_alarms": false_alarms, "sampled_tokens_checked": replays * LM_BATCH,
        "gathered_logits_equal_single_gpu": matches,
    }  # fmt: skip


def e4m3_reading(args, device, steps: int, warmup: int) -> dict:
    """Config 3 at batch 1 on one GPU: the same decode layer with per-row E4M3 weights,
    checked against Q with the fused checker, verdicts carried by the next launch."""
    import copy

    a = copy.copy(args)
    a.weights, a.batch = "e4m3", 1
    groups, _verdict, plain, _xs, ex, _ex_plain, _ = build_layer(a, 0, 1, device)
    for i, g in enumerate(groups):
        g.set_prior([groups[i - 1]])
        if not args.no_prefetch:
            g.set_next(groups[(i + 1) % len(groups)])
    per = graph_steps(steps)
    g_checked = cuda_graph(lambda: [g.launch() for g in groups], per)
    g_plain = cuda_graph(lambda: [g.launch() for g in plain], per)
    g_checked[0].replay()
    torch.cuda.synchronize()
    passed = bool(ex.parts[1].local.all())
    t_checked = timed(g_checked, steps, warmup, 1)
    t_plain = timed(g_plain, steps, warmup, 1)
    per_launch = launch_times([[g.launch for g in groups]], max(10, steps), 1)
    step_bytes = sum(g.algorithmic_bytes for g in groups)
    value = step_bytes / t_checked / 1e9
    peak = float(measured_peaks()["hbm_gbs"])
    del g_checked, g_plain
    return {
        "workload": "llama3-8b decode layer, E4M3 weights (per-row absmax scales) x bf16 activations, batch 1, "
                    "fused blocked check against Q",
        "value": round(value, 2), "unit": UNIT, "ms_per_step": round(t_checked * 1e3, 5),
        "unchecked_ms_per_step": round(t_plain * 1e3, 5),
        "checker_overhead_pct": round((t_checked / t_plain - 1) * 100, 2),
        "launch_ms": per_launch, "all_blocks_passed": passed,
        "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / peak, 4), "traffic": profile_traffic("e4m3"),
                     "scope": "one step = 4 stream_kernel launches (E4M3), each deciding the previous launch's checks"},
    }  # fmt: skip


def batch128_reading(args, groups, device, steps: int, warmup: int) -> dict:
    """The same decode layer (same weights) at a decode batch of 128 on the tensor cores
    (config 2's batched reading): unchecked, and checked with checkers of the tensor-core
    accumulation's declared height. CUDA graphs of one step each, device time."""
    from pck.cuda import GpuBlockedChecker, tc_height
    from pck.cuda.plan import TcLaunch

    gen = torch.Generator().manual_seed(128)
    plain, checked, flops, wbytes = [], [], 0, 0
    for gi, g in enumerate(groups):
        n = g.items[0][0].size(1)
        X = outlier_x(n, 128, gen).to(device).contiguous()
        items_p, items_c = [], []
        for k, (W, _, _) in enumerate(g.items):
            ch = GpuBlockedChecker(W, args.block, tc_height(n), checks=args.checks,
                                   generator=torch.Generator().manual_seed(3000 + 10 * gi + k))  # fmt: skip
            items_p.append((W, X, None))
            items_c.append((W, X, ch))
            flops += 2 * W.numel() * 128
            wbytes += W.numel() * 2
        plain.append(TcLaunch(items_p))
        checked.append(TcLaunch(items_c))
    g_plain = cuda_graph(lambda: [t.launch() for t in plain])
    g_checked = cuda_graph(lambda: [t.launch() for t in checked])
    g_checked[0].replay()
    torch.cuda.synchronize()
    passed = all(bool(r.passed.all()) for t in checked for r in t.results if r is not None)
    t_plain = timed(g_plain, steps, warmup, 1)
    t_checked = timed(g_checked, steps, warmup, 1)
    del g_plain, g_checked
    return {
        "batch": 128, "path": "tcgen05 (tc_kernel) + binary64 bank kernel + verdicts", "all_blocks_passed": passed,
        "unchecked_ms_per_step": round(t_plain * 1e3, 4), "checked_ms_per_step": round(t_checked * 1e3, 4),
        "tokens_per_s_checked": round(128 / t_checked), "tokens_per_s_unchecked": round(128 / t_plain),
        "weight_GB_per_s_unchecked": round(wbytes / t_plain / 1e9, 1),
        "tflops_unchecked": round(flops / t_plain / 1e12, 1),
        "checker_overhead_pct": round((t_checked / t_plain - 1) * 100, 1),
    }  # fmt: skip


def host_layer(args, gpu_groups=None):
    """The layer on the host for the CPU legs: same seeds, same checker banks (copied from
    the GPU when it exists, built on the CPU otherwise)."""
    from oracle.checker import gpu_bank
    from oracle.cpu_baseline import HostMatrix
    from pck.cuda.plan import LLAMA3_8B_GROUPS
    from pck.fp import tree_height

    gen = torch.Generator().manual_seed(0)
    mats, j = [], 0
    for gi, group in enumerate(LLAMA3_8B_GROUPS):
        n = group[0][2]
        x = outlier_x(n, 1, gen)[0]
        for k, (_name, m, nn) in enumerate(group):
            if gpu_groups is not None:
                W, _, ch = gpu_groups[gi].items[k]
                Wc = W.cpu()
                c, a, r = ch.c.cpu().numpy(), ch.a.float().cpu().numpy(), ch.r.cpu().numpy()
                coef, geps, floor = ch.coef, ch.geps, ch.tau_floor
            else:
                Wc = (torch.randn(m, nn, generator=torch.Generator().manual_seed(1000 + j)) * 0.02).bfloat16()
                bank = gpu_bank(Wc, args.block, tree_height(nn, args.threads, 8), args.checks,
                                torch.Generator().manual_seed(2000 + j), segments=1)  # fmt: skip
                c, a, r = bank["c"].numpy(), bank["a"].float().numpy(), bank["r"].numpy()
                coef, geps, floor = bank["coef"], bank["geps"], bank["tau_floor"]
            mats.append(HostMatrix(Wc.view(torch.uint16).numpy(), x.view(torch.uint16).numpy(),
                                   c.astype(np.float64), a.astype(np.float64), r.astype(np.float64),
                                   coef, geps, floor))  # fmt: skip
            j += 1
    return mats


def layer_bytes(mats) -> int:
    total = 0
    for mat in mats:
        m, n = mat.W_bits.shape
        K, nb, _ = mat.c.shape
        total += 2 * m * n + 2 * n + 4 * m + K * nb * n * 4 + nb * n * 2 + mat.r.size + K * nb * 17
    return total


def run_reference(args) -> None:
    """The reference arm: the reference's CPU path (the oracle port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.cpu_baseline import checked_step
    from oracle.gemv import host_threads

    mats = host_layer(args)
    cores = host_threads()
    step_bytes = layer_bytes(mats)
    for _ in range(max(1, args.warmup)):
        checked_step(mats, args.threads, cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        checked_step(mats, args.threads, cores)
    per_step = (time.perf_counter() - t0) / args.steps
    value = step_bytes / per_step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; weights N(0,0.02^2), activations N(0,1) with 1% outliers x20)",
        "config": {"workload": "llama3-8b decode layer GEMV set + blocked check (reference CPU path)",
                   "batch": 1, "block": args.block, "checks": args.checks, "threads": args.threads},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"the whole checked layer, {args.steps} steps (oracle/gemv_ref.c + NumPy check)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }  # fmt: skip
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=50)
    parser.add_argument("--impl", choices=["pck", "reference"], default="pck")
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--block", type=int, default=128)
    parser.add_argument("--checks", type=int, default=1)
    parser.add_argument("--weights", choices=["bf16", "e4m3"], default="bf16",
                        help="weight format (e4m3: config 3, per-row quantised weights)")
    parser.add_argument("--threads", type=int, default=256)
    parser.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample length")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-batch128", action="store_true", help="skip the batch-128 tensor-core reading")
    parser.add_argument("--no-e4m3", action="store_true", help="skip the E4M3 (config 3, batch 1) reading")
    parser.add_argument("--no-lm-head", action="store_true", help="skip the LM-head (config 5) reading")
    parser.add_argument("--no-prefetch", action="store_true",
                        help="launches do not prefetch the next launch's first weight pieces into L2")
    parser.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                        help="N > 1: the all-gather of the outputs (peer: pck_peer_all_gather over NVLink)")
    parser.add_argument("--verdicts", choices=sorted(VERDICTS), default="carried",
                        help="carried: each launch decides the previous launch's checks; launch: a verdict launch per step")
    args = parser.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)  # fmt: skip

    groups, verdict, plain, xs, ex, ex_plain, full = build_layer(args, rank, world, device, keep_full=world > 1)
    x_all = build_layer.x_all
    vs = ex.parts[1]
    step_bytes_local = sum(g.algorithmic_bytes for g in groups)
    # Layer copies in rotation, one per step, so that a rank's weights exceed L2 between reuses
    # (each copy its own memory, the same values, writing the same output buffers).
    copies = layer_copies(step_bytes_local, args.steps)
    layers = [(groups, verdict, plain)]
    share = build_layer.share
    for _ in range(copies - 1):
        g2, v2, p2, *_ = build_layer(args, rank, world, device, share=share)
        layers.append((g2, v2, p2))
    if world > 1 and args.gather == "peer":
        ex.use_peer_memory()
        ex_plain.use_peer_memory()

    def step_of(launches):
        def checked_step() -> None:
            for g in launches:
                g.launch()
            if world > 1:
                ex.gather()

        return checked_step

    # the other verdict form, for comparison (captured before the launches are re-planned)
    per_graph = graph_steps(args.steps, copies)
    graph_other = (cuda_graph(rotation([step_of([*g, v]) for g, v, _ in layers]), per_graph)
                   if args.verdicts == "carried" else None)  # fmt: skip
    chain = [g for gs, _, _ in layers for g in gs]  # every launch of the rotation, in order
    if args.verdicts == "carried":  # each launch decides the previous one's checks
        for i, g in enumerate(chain):
            g.set_prior([chain[i - 1]])
            if not args.no_prefetch:  # and prefetches the next one's first weight pieces
                g.set_next(chain[(i + 1) % len(chain)])
        layer_launches = [list(gs) for gs, _, _ in layers]
    else:
        layer_launches = [[*gs, v] for gs, v, _ in layers]
    launches = layer_launches[0]
    checked_step = rotation([step_of(ls) for ls in layer_launches])
    plain_chain = [g for _, _, ps in layers for g in ps]
    if not args.no_prefetch:
        for i, g in enumerate(plain_chain):
            g.set_next(plain_chain[(i + 1) % len(plain_chain)])

    def plain_of(ps):
        def plain_step() -> None:
            for g in ps:
                g.launch()
            if world > 1:
                ex_plain.gather()

        return plain_step

    def local_of(ls):
        def local_step() -> None:  # the launches alone, without the gather (N > 1 breakdown)
            for g in ls:
                g.launch()

        return local_step

    plain_step = rotation([plain_of(ps) for _, _, ps in layers])
    local_step = rotation([local_of(ls) for ls in layer_launches])

    graph_checked = cuda_graph(checked_step, per_graph)
    graph_plain = cuda_graph(plain_step, per_graph)
    graph_local = cuda_graph(local_step, per_graph) if world > 1 else None
    # correctness of the timed path: every block of the honest layer passes on every rank,
    # and (N > 1) the gathered outputs equal the unsharded ones bit for bit
    graph_checked[0].replay()
    torch.cuda.synchronize()
    all_passed = all_ranks(bool(vs.local.all()), world)
    gathered_ok = gathered_layer_matches(groups, xs, ex, full, world, rank)
    del full

    gpu_index = local
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        try:
            gpu_index = int(visible.split(",")[local])
        except (ValueError, IndexError):
            pass
    with ClockSampler(gpu_index) as clocks:
        t_checked = timed(graph_checked, args.steps, args.warmup, world)
        t_plain = timed(graph_plain, args.steps, args.warmup, world)
        t_other = timed(graph_other, args.steps, args.warmup, world) if graph_other is not None else None
        t_local = timed(graph_local, args.steps, args.warmup, world) if graph_local is not None else None
    clock = clocks.summary()
    side_steps = max(20, args.steps // 10)
    per_launch = launch_times([[g.launch for g in ls] + ([ex.gather] if world > 1 else []) for ls in layer_launches],
                              side_steps, world)  # fmt: skip
    batch128 = e4m3 = lm_head = None
    if world == 1 and args.weights == "bf16" and args.batch == 1 and not args.no_batch128:
        batch128 = batch128_reading(args, groups, device, side_steps, args.warmup)
    if world == 1 and args.weights == "bf16" and args.batch == 1 and not args.no_e4m3:
        e4m3 = e4m3_reading(args, device, side_steps, args.warmup)
    if not args.no_lm_head:
        lm_head = lm_head_reading(rank, world, device, side_steps, args.warmup, args.gather)
    t_e2e, h2d, d2h = e2e_step_time(layer_launches, x_all, ex, side_steps, args.warmup, world)

    total_bytes = torch.tensor([float(step_bytes_local)], device=device)
    if world > 1:
        torch.distributed.all_reduce(total_bytes)
    step_bytes = float(total_bytes.item())
    value = step_bytes / t_checked / 1e9
    peaks = measured_peaks()
    peak = float(peaks["hbm_gbs"])
    traffic = profile_traffic(args.weights)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.weights == "bf16":
        from oracle.cpu_baseline import time_checked_layer

        mats = host_layer(args, groups)
        timing = time_checked_layer(mats, args.threads, min_seconds=args.cpu_seconds, max_steps=10**6)
        cpu_value = layer_bytes(mats) * timing["steps"] / timing["seconds"] / 1e9
        cpu = {"value": round(cpu_value, 3), "unit": UNIT, "cores": timing["cores"], "kind": "port",
               "sample": f"{timing['steps']} whole checked layers in {timing['seconds']:.1f} s "
                         "(oracle/gemv_ref.c over all host threads + NumPy check)"}  # fmt: skip

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_checked * 1e3, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if args.weights == "bf16" else "e4m3 x bf16",
            "data": "synthetic (seeded; weights N(0,0.02^2), activations N(0,1) with 1% outliers x20)",
            "config": {
                "workload": "llama3-8b decode layer GEMV set (q,k,v,o,gate,up,down) + fused blocked check",
                "weights": args.weights,
                "batch": args.batch, "block": args.block, "checks": args.checks, "threads": args.threads,
                "launches_per_step": len(launches),
                "verdicts": VERDICTS[args.verdicts], "parallelism": f"row-shard x{world}" if world > 1 else "single",
                "l2": f"inputs larger than L2: {copies} layer cop{'y' if copies == 1 else 'ies'} in rotation, one per "
                      f"step, {copies * step_bytes_local / 1e6:.0f} MB of weights per rank between reuses, 126 MB L2",
                "layer_copies": copies,
                "graph": f"CUDA graph of {per_graph} consecutive steps, replayed",
                "prefetch": "none" if args.no_prefetch else
                            "each launch's CTAs prefetch the next launch's first weight pieces into L2 as they finish",
            },
            "checker_overhead_pct": round((t_checked / t_plain - 1) * 100, 2),
            "unchecked_ms_per_step": round(t_plain * 1e3, 5),
            "verdict_launch_ms_per_step": round(t_other * 1e3, 5) if t_other is not None else None,
            "all_blocks_passed": all_passed,
            "gathered_outputs_equal_single_gpu": gathered_ok,
            "gather": ex.transport if world > 1 else None,
            "local_launches_ms_per_step": round(t_local * 1e3, 5) if t_local is not None else None,
            "gather_ms_per_step": round((t_checked - t_local) * 1e3, 5) if t_local is not None else None,
            "launch_ms": {"launches": [f"stream_kernel:{'+'.join(grp)}" for grp in LLAMA3_GROUP_NAMES]
                                      + ([f"{ex.transport} all_gather"] if world > 1 else []) + ([] if args.verdicts == "carried"
                                                                                     else ["verdict_kernel"]),
                          "ms": per_launch,
                          "how": "eager, a CUDA event between consecutive launches, mean over "
                                 f"{side_steps} steps, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": round(value / world, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(value / world / peak, 4),
                         "traffic": traffic,
                         "scope": f"one step = {SCOPE[args.verdicts]}; "
                                  "achieved and traffic are per step (ncu summary in profiles/)",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if not peaks.get("fallback") else "fallback"},
            "e2e": {"value": round(step_bytes / t_e2e / 1e9, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(t_e2e * 1e3, 4)},
            "gpu_launches": (len(launches) + (1 if world > 1 and ex.transport == "peer" else 0)) * args.steps,
            "clocks": clock,
            "cpu_baseline": cpu,
            "batch128": batch128,
            "e4m3": e4m3,
            "lm_head": lm_head,
        }  # fmt: skip
        print(json.dumps(line), flush=True)
    del graph_checked, graph_plain, graph_other, graph_local
    if world > 1:
        ex.close()
        ex_plain.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
