"""Device timing on a cold L2 (the reference's src/pck/cuda/timing.py:26-55).

Times are CUDA-event durations on the current stream; before every timed rep a buffer of
twice the L2 size is overwritten (outside the timed region), so weights are read from HBM.
"""

from __future__ import annotations

import re
import statistics
from collections.abc import Callable
from dataclasses import dataclass

import torch


def device_name() -> str:
    return re.sub(r"\s+\w+ GPU$", "", torch.cuda.get_device_name())


@dataclass
class Timing:
    median_ms: float
    p10_ms: float
    p90_ms: float
    mean_ms: float


class ColdL2Timer:
    """Times a CUDA function with events, flushing L2 before every rep."""

    def __init__(self, warmup: int, reps: int) -> None:
        l2 = int(getattr(torch.cuda.get_device_properties(torch.cuda.current_device()), "L2_cache_size", 64 << 20))
        self.flush = torch.empty(2 * max(l2, 1 << 20), dtype=torch.uint8, device="cuda")
        self.warmup, self.reps = warmup, reps

    def __call__(self, fn: Callable[[], object]) -> Timing:
        for _ in range(self.warmup):
            fn()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(self.reps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(self.reps)]
        for start, end in zip(starts, ends, strict=True):
            self.flush.zero_()
            start.record()
            fn()
            end.record()
        torch.cuda.synchronize()
        times = sorted(float(s.elapsed_time(e)) for s, e in zip(starts, ends, strict=True))
        deciles = statistics.quantiles(times, n=10) if len(times) > 1 else [times[0]] * 9
        return Timing(statistics.median(times), deciles[0], deciles[-1], statistics.fmean(times))


def copy_bandwidth_gbps(timer: ColdL2Timer, nbytes: int = 1 << 30) -> float:
    """Device-to-device copy bandwidth (read + write bytes)."""
    src = torch.empty(nbytes // 2, dtype=torch.uint8, device="cuda")
    dst = torch.empty_like(src)
    t = timer(lambda: dst.copy_(src))
    return float(2 * src.numel() / (t.median_ms / 1e3) / 1e9)
