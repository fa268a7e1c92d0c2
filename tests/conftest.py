"""Test configuration: import paths, the `gpu` marker and Hypothesis profiles.

Tests marked `gpu` need a CUDA device and the built library; everything else runs on CPU.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
from hypothesis import HealthCheck, settings

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "proof-carrying-kernels_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

settings.register_profile("default", deadline=None, suppress_health_check=[HealthCheck.too_slow])
settings.register_profile(
    "ci", parent=settings.get_profile("default"), max_examples=300, derandomize=True, print_blob=True
)
settings.load_profile(os.environ.get("HYPOTHESIS_PROFILE", "default"))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU and libpck_b200.so (run with -m gpu)")


def cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()
