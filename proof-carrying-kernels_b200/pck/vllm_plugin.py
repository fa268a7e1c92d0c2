"""Check every token vLLM samples with the fused membership kernel: a vLLM general plugin
(the drop-in for src/pck/vllm_plugin.py; off unless enabled).

vLLM loads entry points of the ``vllm.general_plugins`` group in every process; `register`
does nothing unless ``PCK_CHECK_SAMPLING=1``. Then it wraps the sampler of vLLM's V2 model
runner (vLLM 0.22: ``vllm.v1.worker.gpu.sample``): ``SamplingStates.apply_top_k_top_p`` keeps
the logits as they are before top-k / top-p masking (after penalties and temperature) with the
request's top-k / top-p, and ``Sampler.sample`` checks every sampled token against them with
`pck.member.check_members` (one kernel launch per step, no synchronization: top-k comes from
vLLM's host copy, the counts stay on the device). Every ``PCK_CHECK_EVERY`` steps a JSON line of
running totals (process id, rank) is appended to ``PCK_CHECK_LOG``, one interval late so the
decode loop never waits, and a final line at exit.

Environment:
  PCK_CHECK_SAMPLING=1   enable the check
  PCK_CHECK_LOG          JSON-lines file (default: pck_sampling_check.jsonl)
  PCK_CHECK_EVERY        steps between lines (default 16)
  PCK_CHECK_TOL          the sampler's own top-p tolerance (default 1e-4)
  PCK_FAULT_RATE         fault injection: replace this share of the sampled tokens of
                         constrained rows (top-k, top-p or greedy) with the row's lowest-logit
                         token when that token is outside the allowed set (default 0)
"""

from __future__ import annotations

import atexit
import json
import os
import time
from collections import deque
from pathlib import Path
from typing import Any

import torch

from pck.member import check_members


class SamplingTally:
    """Per-process totals of the sampling check, kept on the device and reported without
    ever stalling the decode loop.

    Each step files every row into one of four bins, ``2 * injected + rejected`` (honest and
    accepted, false alarm, missed injection, caught injection), added in place to a device
    histogram, and folds the step's largest top-p excess into a running maximum. Every
    ``every`` steps both are copied into a pinned host buffer behind an event; the queue of
    such copies is drained (oldest first) whenever their events have completed, so a line is
    written once its copy has arrived and none is dropped. `close` waits for what is still in
    flight and adds a line with the current totals. The JSON-lines schema (rows, rejected,
    injected, caught, false_alarms, steps, max_excess, seconds, pid, rank) is the reference
    plugin's log format."""

    def __init__(self, path: Path, every: int) -> None:
        self.path = path
        self.every = max(1, every)
        self.step = 0
        self.last_reported = 0
        self.bins: torch.Tensor | None = None  # int64 (4,)
        self.peak: torch.Tensor | None = None  # float64 (1,)
        self.inflight: deque[tuple[torch.Tensor, torch.cuda.Event | None, int, float]] = deque()
        self.t0 = time.monotonic()
        self.rank = os.environ.get("RANK", os.environ.get("LOCAL_RANK"))

    def add(self, ok: torch.Tensor, injected: torch.Tensor, excess: torch.Tensor) -> None:
        if self.bins is None:
            self.bins = torch.zeros(4, dtype=torch.int64, device=ok.device)
            self.peak = torch.full((1,), -1.0, dtype=torch.float64, device=ok.device)
        code = injected.to(torch.int64) * 2 + (~ok).to(torch.int64)
        self.bins.index_add_(0, code, torch.ones_like(code))
        torch.maximum(self.peak, excess.max().reshape(1), out=self.peak)
        self.step += 1
        if self.step % self.every == 0:
            self._enqueue()
        self._drain(block=False)

    def _enqueue(self) -> None:
        merged = torch.cat((self.bins.double(), self.peak))
        if merged.is_cuda:
            host = torch.empty(5, dtype=torch.float64, pin_memory=True)
            host.copy_(merged, non_blocking=True)
            done = torch.cuda.Event()
            done.record()
        else:
            host, done = merged.clone(), None
        self.inflight.append((host, done, self.step, time.monotonic() - self.t0))

    def _drain(self, block: bool) -> None:
        while self.inflight:
            host, done, step, elapsed = self.inflight[0]
            if done is not None and not done.query():
                if not block:
                    return
                done.synchronize()
            self.inflight.popleft()
            honest_ok, false_alarm, missed, caught = (int(v) for v in host[:4].tolist())
            line = {"rows": honest_ok + false_alarm + missed + caught, "rejected": false_alarm + caught,
                    "injected": missed + caught, "caught": caught, "false_alarms": false_alarm,
                    "steps": step, "max_excess": float(host[4]), "seconds": round(elapsed, 1),
                    "pid": os.getpid(), "rank": self.rank}  # fmt: skip
            with self.path.open("a") as log:
                log.write(json.dumps(line) + "\n")
            self.last_reported = step

    def close(self) -> None:
        """Write every queued copy and then the current totals (synchronizes; for exit)."""
        self._drain(block=True)
        if self.bins is not None and self.last_reported != self.step:
            self._enqueue()
            self._drain(block=True)


def install(sampler_cls: Any, states_cls: Any, log: Path, every: int = 16, tol: float = 1e-4,
            fault_rate: float = 0.0) -> SamplingTally:  # fmt: skip
    """Wrap ``states_cls.apply_top_k_top_p`` and ``sampler_cls.sample`` (vLLM's V2 sampler
    classes, or stand-ins with the same methods and attributes in tests)."""
    original_mask = states_cls.apply_top_k_top_p
    original_sample = sampler_cls.sample
    stats = SamplingTally(log, every)

    def keep_unmasked(self: Any, logits: torch.Tensor, expanded_idx_mapping: torch.Tensor, idx_mapping_np: Any):
        host_k = self.top_k.np[idx_mapping_np]
        do_top_k = bool((host_k != self.vocab_size).any())
        do_top_p = bool((self.top_p.np[idx_mapping_np] != 1.0).any())
        self._pck_unmasked = (
            logits.clone(),  # vLLM may mask in place
            self.top_k.gpu[expanded_idx_mapping] if do_top_k else None,
            self.top_p.gpu[expanded_idx_mapping] if do_top_p else None,
            host_k if do_top_k else None,
            self.temperature.gpu[expanded_idx_mapping] == 0,
        )
        return original_mask(self, logits, expanded_idx_mapping, idx_mapping_np)

    def checked(self: Any, logits: torch.Tensor, *args: Any, **kwargs: Any):
        states = self.sampling_states
        states._pck_unmasked = None
        sampled, processed = original_sample(self, logits, *args, **kwargs)
        kept = states._pck_unmasked
        if kept is None:  # vLLM skipped the masking step: no top-k / top-p this step
            expanded_idx_mapping = args[0] if args else kwargs["expanded_idx_mapping"]
            kept = (processed, None, None, None, states.temperature.gpu[expanded_idx_mapping] == 0)
        unmasked, top_k, top_p, top_k_host, greedy = kept
        rows, vocab = unmasked.shape
        constrained = greedy.clone()
        if top_k is not None:
            constrained |= top_k < vocab
        if top_p is not None:
            constrained |= top_p < 1.0
        injected = torch.zeros(rows, dtype=torch.bool, device=unmasked.device)
        flat = sampled.reshape(rows)
        if fault_rate > 0:
            draw = torch.rand(rows, device=unmasked.device) < fault_rate
            worst = unmasked.argmin(dim=1).to(flat.dtype)
            legit = check_members(unmasked, worst, top_k, top_p, greedy, tol, top_k_host)["ok"]
            injected = draw & constrained & ~legit
            flat = torch.where(injected, worst, flat)
            sampled = flat.reshape(sampled.shape)
        verdict = check_members(unmasked, flat, top_k, top_p, greedy, tol, top_k_host)
        excess = torch.full((rows,), -1.0, dtype=torch.float64, device=unmasked.device)
        if top_p is not None:  # how close accepted top-p samples come to the boundary
            in_nucleus = verdict["ok"] & (top_p < 1.0) & ~greedy
            excess = torch.where(in_nucleus, verdict["mass_above"] - top_p.double(), excess)
        stats.add(verdict["ok"], injected, excess)
        return sampled, processed

    states_cls.apply_top_k_top_p = keep_unmasked
    sampler_cls.sample = checked
    atexit.register(stats.close)
    return stats


def register() -> None:
    """vLLM's plugin entry point: install the check if ``PCK_CHECK_SAMPLING=1``."""
    if os.environ.get("PCK_CHECK_SAMPLING") != "1":
        return
    from vllm.v1.worker.gpu.sample import sampler as vllm_sampler
    from vllm.v1.worker.gpu.sample import states as vllm_states

    install(vllm_sampler.Sampler, vllm_states.SamplingStates,
            Path(os.environ.get("PCK_CHECK_LOG", "pck_sampling_check.jsonl")),
            every=int(os.environ.get("PCK_CHECK_EVERY", "16")), tol=float(os.environ.get("PCK_CHECK_TOL", "1e-4")),
            fault_rate=float(os.environ.get("PCK_FAULT_RATE", "0")))  # fmt: skip
