"""A short run of the fault-injection campaign (the reference's harness/campaign.py, config 4):
no false alarm on honest outputs of either bit-exact GEMV, and every block with a single wrong
element whose error exceeds 2 tau caught."""

from __future__ import annotations

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def test_short_campaign() -> None:
    from pck.campaign import run

    out = run(inputs=64, batch=16, checks=8, block=128, seed=3, device=torch.device("cuda", 0))
    assert out["honest"]["false_alarms"] == {"coalesced": 0, "naive": 0}
    assert out["honest"]["block_checks"]["coalesced"] == 64 * 32 * 8
    assert max(out["honest"]["max_rho_over_tau"].values()) < 1.0
    for name, t in out["planted"].items():
        assert t["faulty_blocks"] > 0, name
        assert t["single_element_above_2tau_caught"] == t["single_element_above_2tau"], name


def test_short_tensor_core_campaign() -> None:
    """The tensor-core GEMV under its declared height: no false alarm of the fused checks over
    every activation distribution, observed errors inside the declared bound, and every
    single-element fault above 2 tau caught."""
    from pck.campaign import run_tc

    out = run_tc(inputs=512, batch=128, checks=4, block=128, seed=5, device=torch.device("cuda", 0), bound_every=1)
    assert out["honest"]["false_alarms"] == 0
    assert out["honest"]["block_checks"] == 512 * 32 * 4
    assert out["honest"]["max_rho_over_tau"] < 1.0
    assert out["honest"]["max_error_over_declared_bound"] < 1.0
    for name, t in out["planted"].items():
        assert t["faulty_blocks"] > 0, name
        assert t["single_element_above_2tau_caught"] == t["single_element_above_2tau"], name
