"""The bench's step plan (CPU only): how many copies of the layer a rank rotates through so that
its weights exceed L2 between reuses, and how many steps each CUDA graph holds."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

LAYER = 446_729_808  # the checked Llama-3-8B layer's algorithmic bytes at one GPU


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("steps", [20, 50, 100, 400, 2000])
def test_rotation_exceeds_l2_and_graphs_hold_whole_rotations(world: int, steps: int) -> None:
    layer = LAYER // world
    copies = bench.layer_copies(layer, steps)
    per = bench.graph_steps(steps, copies)
    assert copies * layer >= 1.5 * bench.L2_BYTES
    assert steps % per == 0 and per % copies == 0 and per <= bench.GRAPH_STEPS
    need = max(1, -(-int(1.5 * bench.L2_BYTES) // layer))
    for fewer in range(need, copies):  # the count is the smallest that graphs can hold whole
        assert not any(steps % d == 0 and d % fewer == 0 for d in range(fewer, min(steps, bench.GRAPH_STEPS) + 1))


def test_shards_that_fit_in_l2_rotate() -> None:
    assert bench.layer_copies(LAYER, 400) == 1
    assert bench.layer_copies(LAYER // 2, 400) == 1
    assert bench.layer_copies(LAYER // 4, 400) == 2
    assert bench.layer_copies(LAYER // 8, 400) == 4
    assert bench.layer_copies(LAYER // 8, 50) == 5  # no divisor of 50 up to 32 is a multiple of 4


def test_rotation_runs_each_copy_in_turn() -> None:
    seen = []
    step = bench.rotation([lambda i=i: seen.append(i) for i in range(3)])
    for _ in range(7):
        step()
    assert seen == [0, 1, 2, 0, 1, 2, 0]
