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
from pathlib import Path
from typing import Any

import torch

from pck.member import check_members


class CheckStats:
    """Running totals as device tensors; written from pinned host copies, an interval late."""

    FIELDS = ("rows", "rejected", "injected", "caught", "false_alarms")

    def __init__(self, path: Path, every: int) -> None:
        self.path, self.every = path, every
        self.steps = 0
        self.written = 0
        self.totals: torch.Tensor | None = None
        self.max_excess: torch.Tensor | None = None
        self.pending: tuple[torch.Tensor, Any, int, float] | None = None
        self.start = time.time()
        self.rank = os.environ.get("RANK", os.environ.get("LOCAL_RANK"))

    def add(self, ok: torch.Tensor, injected: torch.Tensor, excess: torch.Tensor) -> None:
        rejected = ~ok
        counts = torch.stack([torch.ones_like(ok).sum(), rejected.sum(), injected.sum(),
                              (rejected & injected).sum(), (rejected & ~injected).sum()])  # fmt: skip
        step_excess = excess.max()
        if self.totals is None:
            self.totals, self.max_excess = counts, step_excess
        else:
            self.totals = self.totals + counts
            self.max_excess = torch.maximum(self.max_excess, step_excess)
        self.steps += 1
        if self.steps % self.every == 0:
            self._write_ready(wait=False)
            self.pending = self._snapshot()

    def _snapshot(self) -> tuple[torch.Tensor, Any, int, float]:
        vals = torch.cat([self.totals.to(torch.float64), self.max_excess.reshape(1).double()])
        if not vals.is_cuda:
            return vals.clone(), None, self.steps, time.time()
        host = torch.empty(vals.shape, dtype=vals.dtype, pin_memory=True)
        host.copy_(vals, non_blocking=True)
        event = torch.cuda.Event()
        event.record()
        return host, event, self.steps, time.time()

    def _write_ready(self, wait: bool) -> None:
        if self.pending is None:
            return
        host, event, steps, now = self.pending
        if event is not None and not event.query():
            if not wait:
                return  # still in flight: the next snapshot replaces it
            event.synchronize()
        values = host.tolist()
        row: dict[str, Any] = dict(zip(self.FIELDS, (int(v) for v in values[:-1]), strict=True))
        row |= {"steps": steps, "max_excess": values[-1], "seconds": round(now - self.start, 1),
                "pid": os.getpid(), "rank": self.rank}  # fmt: skip
        with self.path.open("a") as f:
            f.write(json.dumps(row) + "\n")
        self.pending, self.written = None, steps

    def flush(self) -> None:
        """Write the pending copy, then the current totals (synchronizes; for the end)."""
        self._write_ready(wait=True)
        if self.totals is not None and self.written != self.steps:
            self.pending = self._snapshot()
            self._write_ready(wait=True)


def install(sampler_cls: Any, states_cls: Any, log: Path, every: int = 16, tol: float = 1e-4,
            fault_rate: float = 0.0) -> CheckStats:  # fmt: skip
    """Wrap ``states_cls.apply_top_k_top_p`` and ``sampler_cls.sample`` (vLLM's V2 sampler
    classes, or stand-ins with the same methods and attributes in tests)."""
    original_mask = states_cls.apply_top_k_top_p
    original_sample = sampler_cls.sample
    stats = CheckStats(log, every)

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
    atexit.register(stats.flush)
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
