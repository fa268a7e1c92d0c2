"""The checked decode layer on the host cores — the timed CPU baseline and the reference arm
of bench.py. Test infrastructure (a port of the reference's CPU path), never the product.

A step computes, for every projection of the layer, y = W x with the reference's
coalesced tree (oracle/gemv_ref.c, rows split over all host threads) and then the
blocked check of y against the same bank the GPU uses (binary64 NumPy/BLAS:
rho = c.x - r.y, s = a.|x|, tau by the reference's formula). This is the work of the
reference's CPU models `emulate_gemv_coalesced` (src/pck/gemv.py:71-101) and
`BlockedChecker.verdict` (src/pck/checker.py:75-99), run with every host thread.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np

from oracle.gemv import gemv_coalesced_c, host_threads

U32 = 2.0**-24


@dataclass
class HostMatrix:
    W_bits: np.ndarray  # (m, n) uint16 bfloat16 bits
    x_bits: np.ndarray  # (n,) uint16
    c: np.ndarray  # (K, nb, n) float64 (binary32 values)
    a: np.ndarray  # (nb, n) float64 (bfloat16 values)
    r: np.ndarray  # (K, nb, b) float64 +-1
    coef: float
    geps: float
    tau_floor: float


def checked_step(mats: list[HostMatrix], threads: int, cpu_threads: int) -> list[np.ndarray]:
    """One checked layer on the CPU; returns each projection's per-block verdicts."""
    verdicts = []
    for mat in mats:
        y = gemv_coalesced_c(mat.W_bits, mat.x_bits, threads, 8, cpu_threads=cpu_threads)
        x = (mat.x_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        K, nb, _ = mat.c.shape
        yb = y.astype(np.float64).reshape(nb, -1)
        rho = mat.c @ x - np.einsum("kbi,bi->kb", mat.r, yb)
        s = mat.a @ np.abs(x)
        tau = mat.coef * s + mat.geps * ((1 + U32) * s + np.abs(yb).sum(axis=1)) + mat.tau_floor
        ok = np.isfinite(yb).all(axis=1) & np.isfinite(tau) & (np.abs(rho) <= tau).all(axis=0)
        verdicts.append(ok)
    return verdicts


def time_checked_layer(mats: list[HostMatrix], threads: int = 256, min_seconds: float = 10.0,
                       max_steps: int = 50, cpu_threads: int | None = None) -> dict:  # fmt: skip
    """Times whole checked steps until ``min_seconds`` of CPU work (at least one step)."""
    cores = cpu_threads or host_threads()
    checked_step(mats, threads, cores)  # warm-up (page-in, thread pool)
    steps, t0 = 0, time.perf_counter()
    while True:
        checked_step(mats, threads, cores)
        steps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= min_seconds or steps >= max_steps:
            break
    return {"steps": steps, "seconds": elapsed, "cores": cores}
