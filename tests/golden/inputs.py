"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Only NumPy and torch (CPU) are used here, so the same arrays come out in the build
container (where the fixtures were generated from the reference's own code) and on a GPU
box. Every fixture also stores a SHA-256 of its inputs, which the tests check first.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch


def bf16_round(a: np.ndarray) -> np.ndarray:
    """binary32 -> bfloat16 (round to nearest even) -> binary32, via torch."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).bfloat16().float().numpy()


def bits16(a: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns of binary32 values that are already bfloat16."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def from_bits16(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def numpy_problem(m: int, n: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """W ~ N(0, 0.02^2), x ~ N(0, 1), both rounded to bfloat16, from default_rng(seed)
    (the convention of the reference's GPU tests, tests/gpu/test_gemv_cuda.py:117-119)."""
    rng = np.random.default_rng(seed)
    return bf16_round(rng.standard_normal((m, n)) * 0.02), bf16_round(rng.standard_normal(n))


def torch_problem(m: int, n: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The same from a CPU torch.Generator (tests/gpu/test_gemv_fp8.py:21-25 and the
    harness benches): bfloat16 CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(m, n, generator=g) * 0.02).bfloat16()
    x = torch.randn(n, generator=g).bfloat16()
    return W, x


FP8_MAX = 448.0


def quantize_fp8_cpu(W: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row absmax/448 E4M3 quantisation, written out for CPU tensors
    (src/pck/cuda/gemv.py:41-48)."""
    amax = W.abs().amax(dim=1).float()
    s = torch.where(amax > 0, amax / FP8_MAX, torch.ones_like(amax))
    Q = (W.float() / s[:, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return Q.contiguous(), s


def fp8_bit_patterns(m: int, n: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Raw E4M3 patterns (every finite value, subnormals included; the NaN pattern
    S.1111.111 replaced by 0) and bfloat16 x of spread magnitudes
    (tests/gpu/test_gemv_fp8.py:39-50)."""
    g = torch.Generator().manual_seed(seed)
    bits = torch.randint(0, 256, (m, n), generator=g, dtype=torch.uint8)
    bits[(bits & 0x7F) == 0x7F] = 0
    x = torch.randn(n, generator=g) * 2.0 ** torch.randint(-8, 8, (n,), generator=g)
    return bits.view(torch.float8_e4m3fn), x.bfloat16()


def outlier_activations(n: int, gen: torch.Generator, scale: float = 20.0) -> torch.Tensor:
    """x ~ N(0, 1) with 1% of channels scaled by ``scale``, as bfloat16 (the decode-layer
    configuration's activations)."""
    x = torch.randn(n, generator=gen)
    idx = torch.randperm(n, generator=gen)[: max(1, n // 100)]
    x[idx] *= scale
    return x.bfloat16()


def member_case_ties(seed: int = 0):
    """Rows with ties at the top, tokens near the top, mixed top-k / top-p / greedy
    (tests/test_member.py:85-112)."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((64, 500)) * 3
    logits[:, :5] = 7.0
    tokens = rng.integers(0, 500, 64)
    tokens[:32] = np.argsort(-logits[:32], axis=1)[np.arange(32), rng.integers(0, 20, 32)]
    top_k = rng.choice([1, 5, 20, 500], 64)
    top_p = rng.choice([0.3, 0.9, 1.0], 64)
    greedy = rng.random(64) < 0.1
    return logits.astype(np.float32), tokens.astype(np.int64), top_k.astype(np.int64), top_p, greedy


def member_case_kth_ties(seed: int = 1):
    """30 tokens tied at the k-th logit in every other row (tests/test_member.py:116-145)."""
    rng = np.random.default_rng(seed)
    rows, vocab = 48, 400
    logits = (rng.standard_normal((rows, vocab)) * 4).astype(np.float32)
    top_k = rng.choice([1, 3, 10, 40], rows)
    for i in range(0, rows, 2):
        order = np.argsort(-logits[i])
        logits[i, order[top_k[i] - 1 : top_k[i] + 29]] = logits[i, order[top_k[i] - 1]]
    tokens = np.array(
        [np.argsort(-row)[rng.integers(0, k)] for row, k in zip(logits, top_k, strict=True)]
    )
    tokens[::5] = rng.integers(0, vocab, len(tokens[::5]))
    top_p = rng.choice([0.2, 0.6, 0.95], rows)
    return logits, tokens.astype(np.int64), top_k.astype(np.int64), top_p


def member_case_wide(seed: int = 2):
    """Logits spread over hundreds of units (tests/test_member.py:148-166)."""
    rng = np.random.default_rng(seed)
    rows, vocab = 16, 5000
    logits = rng.uniform(-300, 40, (rows, vocab)).astype(np.float32)
    logits[:, :50] = rng.uniform(30, 40, (rows, 50)).astype(np.float32)
    tokens = np.argsort(-logits, axis=1)[:, 7]
    return logits, tokens.astype(np.int64)


def member_case_lm_head(rows: int, vocab: int, seed: int, fault_rate: float = 0.01):
    """Config-5 style sampling batch: logits ~ N(0, 3^2), temperature 1, top-k 50,
    top-p 0.9; the sampled token is drawn inside the top-k nucleus, and a ``fault_rate``
    share of rows get the row's argmin token instead (a non-member)."""
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(rows, vocab, generator=g) * 3.0
    k, p = 50, 0.9
    vals, idx = torch.topk(logits, k, dim=1)
    probs = torch.softmax(vals.double(), dim=1)
    cum = torch.cumsum(probs, dim=1)
    keep = (cum - probs) < p  # smallest prefix whose mass reaches p
    probs = torch.where(keep, probs, torch.zeros_like(probs))
    pick = torch.multinomial(probs.float(), 1, generator=g).squeeze(1)
    tokens = idx.gather(1, pick[:, None]).squeeze(1)
    faulty = torch.rand(rows, generator=g) < fault_rate
    tokens = torch.where(faulty, logits.argmin(dim=1), tokens)
    top_k = torch.full((rows,), k, dtype=torch.int64)
    top_p = torch.full((rows,), p, dtype=torch.float64)
    return logits, tokens, top_k, top_p, faulty


def sampling_logits(rows: int, vocab: int, seed: int, scale: float = 3.0, ties: bool = False):
    """tests/gpu/test_sampling_cuda.py:23-30."""
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((rows, vocab)) * scale).astype(np.float32)
    if ties:
        a = bf16_round(a)
    return a
