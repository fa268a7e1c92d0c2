"""The vLLM plugin (the reference's tests/test_vllm_plugin.py, restated): off unless enabled,
wraps vLLM 0.22's V2 sampler, and on a stand-in sampler with the same methods it raises no
false alarm on legitimately sampled tokens and catches every injected non-member."""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch


def test_register_is_off_unless_enabled(monkeypatch) -> None:
    from pck import vllm_plugin

    monkeypatch.delenv("PCK_CHECK_SAMPLING", raising=False)
    assert vllm_plugin.register() is None  # returns before importing vLLM


def test_install_wraps_vllm_v2_sampler(tmp_path: Path) -> None:
    pytest.importorskip("vllm")
    from vllm.v1.worker.gpu.sample import sampler as vs
    from vllm.v1.worker.gpu.sample import states as vst

    from pck import vllm_plugin

    before = (vs.Sampler.sample, vst.SamplingStates.apply_top_k_top_p)
    try:
        vllm_plugin.install(vs.Sampler, vst.SamplingStates, tmp_path / "log.jsonl")
        assert vs.Sampler.sample is not before[0]
        assert vst.SamplingStates.apply_top_k_top_p is not before[1]
    finally:
        vs.Sampler.sample, vst.SamplingStates.apply_top_k_top_p = before


class _Uva:
    """vLLM's UvaBackedTensor in miniature: a host array and its device copy."""

    def __init__(self, values: np.ndarray) -> None:
        self.np = values
        self.gpu = torch.from_numpy(values).cuda()


class _States:
    def __init__(self, vocab: int, top_k: np.ndarray, top_p: np.ndarray, temperature: np.ndarray) -> None:
        self.vocab_size = vocab
        self.top_k = _Uva(top_k.astype(np.int32))
        self.top_p = _Uva(top_p.astype(np.float32))
        self.temperature = _Uva(temperature.astype(np.float32))

    def apply_top_k_top_p(self, logits, expanded_idx_mapping, idx_mapping_np):
        """Mask to the top-k, then to the smallest prefix whose softmax mass reaches top-p."""
        k = self.top_k.gpu[expanded_idx_mapping].long()
        p = self.top_p.gpu[expanded_idx_mapping].double()
        vals, order = torch.sort(logits, dim=1, descending=True)
        rank = torch.arange(logits.size(1), device=logits.device)[None]
        keep = rank < k[:, None]
        probs = torch.softmax(torch.where(keep, vals, torch.full_like(vals, -np.inf)).double(), dim=1)
        before = torch.cumsum(probs, dim=1) - probs
        keep &= before < p[:, None]
        masked = torch.full_like(logits, -np.inf)
        masked.scatter_(1, order, torch.where(keep, vals, torch.full_like(vals, -np.inf)))
        return masked


class _Sampler:
    def __init__(self, states: _States, gen: torch.Generator) -> None:
        self.sampling_states = states
        self.gen = gen

    def sample(self, logits, expanded_idx_mapping, idx_mapping_np, pos, input_ids, expanded_local_pos):
        temp = self.sampling_states.temperature.gpu[expanded_idx_mapping]
        greedy = temp == 0
        scaled = torch.where(greedy[:, None], logits, logits / temp.clamp(min=1e-6)[:, None])
        masked = self.sampling_states.apply_top_k_top_p(scaled, expanded_idx_mapping, idx_mapping_np)
        drawn = torch.multinomial(torch.softmax(masked, dim=1), 1, generator=self.gen).squeeze(1)
        sampled = torch.where(greedy, masked.argmax(dim=1), drawn)
        return sampled, masked


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")
def test_stand_in_sampler_no_false_alarm_and_faults_caught(tmp_path: Path) -> None:
    from pck import vllm_plugin

    rows, vocab = 32, 32000
    rng = np.random.default_rng(0)
    states = _States(vocab, rng.choice([20, 50, vocab], rows), rng.choice([0.8, 0.95, 1.0], rows),
                     rng.choice([0.0, 0.7, 1.0], rows))  # fmt: skip
    log = tmp_path / "log.jsonl"
    stats = vllm_plugin.install(_Sampler, _States, log, every=4, tol=1e-4, fault_rate=0.05)
    sampler = _Sampler(states, torch.Generator("cuda").manual_seed(1))
    idx = torch.arange(rows, device="cuda")
    for step in range(24):
        logits = torch.randn(rows, vocab, device="cuda") * 3.0
        sampler.sample(logits, idx, np.arange(rows), None, None, None)
    stats.close()
    last = json.loads(log.read_text().strip().splitlines()[-1])
    assert last["steps"] == 24 and last["rows"] == 24 * rows
    assert last["false_alarms"] == 0
    assert last["injected"] > 0 and last["caught"] == last["injected"]


def test_tally_lines_on_the_host(tmp_path: Path) -> None:
    """The tally's bins and log lines, driven with host tensors (no GPU): every interval
    writes one line of running totals, and close() adds the unreported tail."""
    from pck.vllm_plugin import SamplingTally

    log = tmp_path / "tally.jsonl"
    tally = SamplingTally(log, every=2)
    steps = [
        (torch.tensor([True, False, True, False]), torch.tensor([False, False, True, True]), torch.tensor([-1.0, 0.2])),
        (torch.tensor([True, True, True, True]), torch.tensor([False, False, False, False]), torch.tensor([0.5, -1.0])),
        (torch.tensor([False, True, True, True]), torch.tensor([True, False, False, False]), torch.tensor([0.1])),
    ]  # fmt: skip
    for ok, injected, excess in steps:
        tally.add(ok, injected, excess.double())
    tally.close()
    lines = [json.loads(x) for x in log.read_text().splitlines()]
    assert [ln["steps"] for ln in lines] == [2, 3]
    first, last = lines
    assert (first["rows"], first["rejected"], first["injected"], first["caught"], first["false_alarms"]) == (8, 2, 2, 1, 1)
    assert (last["rows"], last["rejected"], last["injected"], last["caught"], last["false_alarms"]) == (12, 3, 3, 2, 1)
    assert first["max_excess"] == 0.5 and last["max_excess"] == 0.5
    assert all(ln["pid"] == os.getpid() for ln in lines)
