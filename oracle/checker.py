"""Blocked checksum checker, CPU oracle. Test infrastructure only.

Three restatements of the reference:

1. `WeightBank` / `BlockedChecker` — the reference's CPU checker with NumPy sign draws
   (src/pck/checker.py:11-99).
2. `gpu_bank` — the bank the reference's GPU checker builds at weight load: signs drawn
   with a CPU torch.Generator, c = r^T W_beta in binary64 rounded to binary32, a = sum |W_i|
   rounded up to bfloat16, and the host constants coef, geps, tau_floor, segments
   (src/pck/cuda/checker.py:29-43, 72-129).
3. `gpu_verdict` — the GPU checker's decision rule (src/pck/cuda/csrc/checker_kernel.cu:
   87-185) evaluated with exact arithmetic: rho is the correctly rounded exact residual
   c.x - r.y; the parts of tau that the kernel bounds from above (a.|x| and sum |y|) are
   replaced by the smallest binary64 upper bounds of their exact values; tau then follows
   checker_kernel.cu:176-183 with every operation rounded upward; when a.|x| exceeds the
   binary32 range, where the reference's binary32 bound sums overflow, tau is infinite
   and the block fails closed (reference tests/gpu/test_checker_cuda.py:241-252). Any sound GPU
   implementation returns a tau at least this large and a rho within its own rounding of
   this one, so verdicts agree except within that rounding of |rho| = tau.
"""

from __future__ import annotations

import math
from fractions import Fraction

import numpy as np

from oracle.fp import U32, U64, ceil_div, gamma, next_up, round_up_f32, sum_up, sum_up_factor

# ---------------------------------------------------------------------------------------
# 1. CPU checker with NumPy signs (src/pck/checker.py)


class WeightBank:
    """binary64 blocks of W and a_beta = sum_{i in beta} |W_i| rounded up to binary32
    (src/pck/checker.py:11-24)."""

    def __init__(self, W: np.ndarray, block: int) -> None:
        m, n = W.shape
        if block < 1 or m % block:
            raise ValueError(f"block={block} must be positive and divide m={m}")
        self.shape, self.block = (m, n), block
        self.W_blocks = W.reshape(m // block, block, n).astype(np.float64)
        with np.errstate(over="ignore", invalid="ignore"):
            self.a_up = round_up_f32(sum_up(np.abs(self.W_blocks).sum(axis=1), block))


class BlockedChecker:
    """One random checksum per block (src/pck/checker.py:27-99):
    rho = (r^T W_beta).x - r.y_beta, tau = (gamma_h + u) a.|x| + eps, both binary64;
    a block passes iff all its outputs are finite, tau is finite and |rho| <= tau."""

    def __init__(self, W, x, block: int, height: int, bank: WeightBank | None = None) -> None:
        m, n = W.shape
        if x.shape != (n,):
            raise ValueError(f"x has shape {x.shape}, expected ({n},)")
        if bank is None:
            bank = WeightBank(W, block)
        elif bank.shape != (m, n) or bank.block != block:
            raise ValueError("the weight bank was built for another W or block")
        self.m, self.n, self.block = m, n, block
        self.num_blocks = m // block
        self.W_blocks = bank.W_blocks
        self.x = x.astype(np.float64)
        with np.errstate(over="ignore", invalid="ignore"):
            self.abs_bound = sum_up(bank.a_up @ np.abs(self.x), n)
        self.gamma_h = gamma(height)
        self.coef = next_up(next_up(self.gamma_h) + U32)

    @property
    def tau_base(self) -> np.ndarray:
        with np.errstate(over="ignore", invalid="ignore"):
            return np.nextafter(self.coef * self.abs_bound, np.inf)

    def verdict(self, y, rng: np.random.Generator, checks: int = 1) -> np.ndarray:
        if y.shape != (self.m,):
            raise ValueError(f"y has shape {y.shape}, expected ({self.m},)")
        with np.errstate(invalid="ignore", over="ignore"):
            yb = y.astype(np.float64).reshape(self.num_blocks, self.block)
        ok = np.isfinite(yb).all(axis=1)
        for _ in range(checks):
            r = rng.choice([-1.0, 1.0], (self.num_blocks, self.block))
            c = np.einsum("kb,kbn->kn", r, self.W_blocks).astype(np.float32).astype(np.float64)
            with np.errstate(invalid="ignore", over="ignore"):
                rho = c @ self.x - (r * yb).sum(axis=1)
                mags = sum_up(np.abs(c) @ np.abs(self.x), self.n) + sum_up(
                    np.abs(yb).sum(axis=1), self.block
                )
                eps = np.nextafter(next_up(gamma(self.n + self.block + 1, U64)) * mags, np.inf)
                tau = np.nextafter(self.tau_base + eps, np.inf)
                ok &= np.isfinite(tau) & (np.abs(rho) <= tau)
        return ok


# ---------------------------------------------------------------------------------------
# 2. The GPU checker's bank (src/pck/cuda/checker.py)

KERNEL_THREADS = 256  # threads per block of the reference checker kernel (checker.py:229)
BLOCKS_PER_SM = 4  # checker.py:230
MIN_SEGMENT_COLUMNS = 2 * KERNEL_THREADS  # checker.py:231


def round_up_bf16(v):
    """binary64 -> bfloat16 never rounding down (src/pck/cuda/checker.py:29-43): first up to
    binary32, then up to bfloat16 by carrying into bit 16 when any low bit is set."""
    import torch

    if v.dtype != torch.float64:
        raise TypeError(f"round_up_bf16 expects float64, got {v.dtype}")
    if bool((v < 0).any()):
        raise ValueError("round_up_bf16 expects non-negative values")
    f = v.float()
    f = torch.where(f.double() < v, torch.nextafter(f, torch.full_like(f, math.inf)), f)
    bits = f.view(torch.int32)
    low = (bits & 0xFFFF) != 0
    bits = torch.where(low, (bits + 0x10000) & -0x10000, bits)
    return bits.view(torch.float32).to(torch.bfloat16)


def default_segments(n: int, checks: int, num_blocks: int, sms: int) -> int:
    """checker.py:313-316."""
    wanted = ceil_div(BLOCKS_PER_SM * sms, checks * num_blocks)
    return max(1, min(wanted, n // MIN_SEGMENT_COLUMNS))


def host_constants(n: int, block: int, height: int, segments: int) -> tuple[float, float, float]:
    """(coef, geps, tau_floor) exactly as checker.py:311 and 320-330 compute them."""
    coef = next_up(gamma(height) + U32, 2)
    chain = ceil_div(ceil_div(n, segments), KERNEL_THREADS)
    g2 = gamma(2 * chain, U32) ** 2
    fp64_height = max(n + block + 1, 21 + segments + ceil_div(block, KERNEL_THREADS))
    gh = gamma(fp64_height, U64)
    geps = next_up(gh + g2 + gh * g2, 4)
    tau_floor = next_up(n * 2.0**-148, 2)
    return coef, geps, tau_floor


def gpu_bank(W, block: int, height: int, checks: int = 1, generator=None, segments=None,
             sms: int = 148) -> dict:  # fmt: skip
    """The bank of GpuBlockedChecker(W, block, height, checks, generator, segments), built on
    the CPU from a bfloat16 CPU tensor W (src/pck/cuda/checker.py:72-129)."""
    import torch

    if not (W.dtype == torch.bfloat16 and W.dim() == 2):
        raise ValueError("W must be a 2-D bfloat16 tensor")
    m, n = W.shape
    if block < 1 or m % block:
        raise ValueError(f"block={block} must be positive and divide m={m}")
    if checks < 1:
        raise ValueError(f"checks must be positive, got {checks}")
    nb = m // block
    bits = torch.randint(0, 2, (checks, nb, block), generator=generator)
    r = (2 * bits - 1).to(torch.int8)
    W64 = W.reshape(nb, block, n).double()
    c = torch.stack([torch.einsum("bi,bin->bn", r[k].double(), W64).float() for k in range(checks)])
    col = W64.abs().sum(dim=1) * sum_up_factor(block)
    a = round_up_bf16(torch.nextafter(col, torch.full_like(col, math.inf)))
    if segments is None:
        segments = default_segments(n, checks, nb, sms)
    if not 1 <= segments <= min(n, 65535):
        raise ValueError(f"segments must be in [1, {min(n, 65535)}], got {segments}")
    coef, geps, tau_floor = host_constants(n, block, height, segments)
    return {"r": r, "c": c, "a": a, "coef": coef, "geps": geps, "tau_floor": tau_floor,
            "segments": segments}  # fmt: skip


# ---------------------------------------------------------------------------------------
# 3. The GPU checker's decision rule, exactly


def _round_up(q: Fraction) -> float:
    """Smallest binary64 value >= q (q finite)."""
    f = float(q)
    if math.isinf(f):
        return f
    if Fraction(f) < q:
        f = math.nextafter(f, math.inf)
    return f


def _ru_sum(terms: np.ndarray) -> float:
    """Smallest binary64 value >= the exact sum of ``terms`` (finite binary64 values).

    math.fsum returns the exact sum rounded to nearest; the sign of the exact residual
    (exact sum - that value), which fsum also returns exactly, says whether it fell below.
    """
    t = np.asarray(terms, dtype=np.float64).ravel()
    f = math.fsum(t)
    if math.isinf(f):
        return f
    if math.fsum(np.concatenate([t, [-f]])) > 0:
        f = math.nextafter(f, math.inf)
    return f


def _ru_mul(a: float, b: float) -> float:
    if math.isinf(a) or math.isinf(b) or math.isnan(a) or math.isnan(b):
        return a * b
    return _round_up(Fraction(a) * Fraction(b))


def _ru_add(a: float, b: float) -> float:
    if math.isinf(a) or math.isinf(b) or math.isnan(a) or math.isnan(b):
        return a + b
    return _round_up(Fraction(a) + Fraction(b))


ONE_PLUS_U32 = 1.0 + U32  # exact in binary64
FLOAT_MAX = float(np.finfo(np.float32).max)


def gpu_verdict(c: np.ndarray, a: np.ndarray, r: np.ndarray, x: np.ndarray, y: np.ndarray,
                coef: float, geps: float, tau_floor: float) -> dict:  # fmt: skip
    """Exact-arithmetic evaluation of checker_kernel.cu:87-185 for one GEMV output.

    c (K, nb, n) binary32, a (nb, n) bfloat16 values as binary32, r (K, nb, b) +-1,
    x (n,) bfloat16 values, y (nb*b,) binary32. Returns passed (K, nb) bool, rho (K, nb)
    (correctly rounded exact residual), tau (K, nb) (the least tau a sound implementation
    can produce) and s (nb,) (the least binary64 upper bound of a.|x|).
    """
    K, nb, n = c.shape
    b = r.shape[2]
    x64 = np.asarray(x, dtype=np.float64)
    y64 = np.asarray(y, dtype=np.float64).reshape(nb, b)
    finite = np.isfinite(y64).all(axis=1)
    passed = np.zeros((K, nb), dtype=bool)
    rho = np.zeros((K, nb))
    tau = np.zeros((K, nb))
    s_up = np.zeros(nb)
    absx = np.abs(x64)
    for beta in range(nb):
        # a (8 significant bits) * |x| (8 bits) is exact in binary64
        s = _ru_sum(a[beta].astype(np.float64) * absx)
        s_up[beta] = s
        yb = y64[beta]
        if finite[beta]:
            yabs = _ru_sum(np.abs(yb))
        else:
            yabs = math.inf
        cabs = _ru_mul(ONE_PLUS_U32, s)
        eps = _ru_mul(geps, _ru_add(cabs, yabs))
        t = _ru_add(_ru_add(_ru_mul(coef, s), eps), tau_floor)
        if not s <= FLOAT_MAX:
            # a.|x| beyond binary32: the checked kernel's no-overflow hypothesis fails, and the
            # reference's binary32 bound sums overflow to inf: fail closed
            t = math.inf
        for k in range(K):
            cx = c[k, beta].astype(np.float64) * x64  # binary32 * bfloat16: exact in binary64
            if finite[beta]:
                ry = r[k, beta].astype(np.float64) * yb
                rh = math.fsum(np.concatenate([cx, -ry]))
            else:
                rh = math.nan
            rho[k, beta] = rh
            tau[k, beta] = t
            passed[k, beta] = bool(finite[beta] and math.isfinite(t) and abs(rh) <= t)
    return {"passed": passed, "rho": rho, "tau": tau, "s": s_up}
