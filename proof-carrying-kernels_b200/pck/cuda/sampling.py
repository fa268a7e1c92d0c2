"""Trusted top-k / top-p set checker on the GPU, and untrusted GPU samplers to test it
(the drop-in for src/pck/cuda/sampling.py).

The checker (`check_topk_gpu`, `check_topp_gpu`) runs `pck_sampling_check`: exact binary32
comparisons for the top-k prefix property and binary64 masses for top-p minimality, one
launch for a batch of rows, with selections given as (B, L) int64 tensors and per-row
lengths. The samplers (`topk_sample`, `topp_select`, `sharded_topk_gpu`) are plain torch
code under test, not trusted.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from pck.cuda import _lib
from pck.cuda._ext import on_device, stream_handle
from pck.fp import U32, U64, ceil_div, gamma

BLOCKS_PER_SM = 4
MIN_SEGMENT = 4096  # logits per segment, at least


@dataclass(frozen=True)
class SamplingCheck:
    """Per-row checker outputs, each of shape (B,)."""

    passed: torch.Tensor
    min_selected: torch.Tensor
    max_rejected: torch.Tensor
    mass: torch.Tensor
    mass_without_smallest: torch.Tensor


def default_segments(logits: torch.Tensor) -> int:
    """About ``BLOCKS_PER_SM`` CTAs per SM over the batch, at least MIN_SEGMENT logits each
    (the kernel caps the split of a row at one cluster of 8 CTAs)."""
    rows, vocab = logits.shape
    sms = torch.cuda.get_device_properties(logits.device).multi_processor_count
    return max(1, min(ceil_div(BLOCKS_PER_SM * sms, rows), ceil_div(vocab, MIN_SEGMENT)))


def _check_tensor(t: torch.Tensor, name: str, dtype: torch.dtype, device: torch.device) -> None:
    if not (t.is_cuda and t.device == device):
        raise RuntimeError(f"{name} must be on {device}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _run(logits, selected, lengths, k: int, top_p: bool, p: float, temperature: float, slack: float,
         segments: int) -> SamplingCheck:  # fmt: skip
    if not logits.is_cuda:
        raise RuntimeError("logits must be a CUDA tensor")
    dev = logits.device
    _check_tensor(logits, "logits", torch.float32, dev)
    _check_tensor(selected, "selected", torch.int64, dev)
    _check_tensor(lengths, "lengths", torch.int64, dev)
    if not (logits.dim() == 2 and selected.dim() == 2 and lengths.dim() == 1):
        raise RuntimeError("expected logits (B, V), selected (B, L), lengths (B,)")
    rows, vocab = logits.shape
    if selected.size(0) != rows or lengths.size(0) != rows:
        raise RuntimeError("batch sizes differ")
    out = (torch.empty(rows, dtype=torch.bool, device=dev), torch.empty(rows, dtype=torch.float32, device=dev),
           torch.empty(rows, dtype=torch.float32, device=dev), torch.empty(rows, dtype=torch.float64, device=dev),
           torch.empty(rows, dtype=torch.float64, device=dev))  # fmt: skip
    with on_device(dev):
        rc = _lib.library().pck_sampling_check(
            logits.data_ptr(), selected.data_ptr(), lengths.data_ptr(), rows, vocab, selected.size(1), k,
            int(top_p), p, temperature, slack, segments, *(t.data_ptr() for t in out), stream_handle(dev))
    _lib.check(rc, "sampling checker")
    return SamplingCheck(*out)


def check_topk_gpu(logits: torch.Tensor, selected: torch.Tensor, k: int, segments: int | None = None) -> SamplingCheck:
    """Check that each row of ``selected`` (B, k) is a valid top-k set of ``logits`` (B, V)."""
    segs = default_segments(logits) if segments is None else segments
    lengths = torch.full((selected.shape[0],), selected.shape[1], dtype=torch.int64, device=selected.device)
    return SamplingCheck(*torch.ops.pck.sampling_check(logits, selected, lengths, k, False, 1.0, 1.0, 0.0, segs))


def check_topp_gpu(logits: torch.Tensor, selected: torch.Tensor, lengths: torch.Tensor, p: float,
                   temperature: float = 1.0, tol: float = 1e-6, segments: int | None = None) -> SamplingCheck:  # fmt: skip
    """Check that ``selected[b, :lengths[b]]`` is a valid, minimal top-p nucleus of row b.

    ``tol`` is the sampler's declared probability error; the checker adds its own rounding
    slack, the reference's bound (src/pck/cuda/sampling.py:62-90): every term from binary32
    expf on a split argument is within 6 u32 relative plus 2^-148 absolute, the sums are
    binary64, so each mass is within 16 u32 + V 2^-146 + gamma_{V+3S+16}(u64) (S segments).
    This kernel takes every term against the row maximum and rescales nothing, so the same
    slack covers it with room to spare.
    """
    if not 0 < p <= 1:
        raise ValueError(f"p must be in (0, 1], got {p}")
    if tol < 0:
        raise ValueError(f"tol must be non-negative, got {tol}")
    segs = default_segments(logits) if segments is None else segments
    vocab = logits.shape[1]
    own = 16 * U32 + math.ldexp(vocab, -146) + gamma(vocab + 3 * segs + 16, U64)
    slack = math.nextafter(tol + own, math.inf)
    return SamplingCheck(*torch.ops.pck.sampling_check(logits, selected, lengths, 0, True, p, temperature, slack, segs))


def topk_sample(logits: torch.Tensor, k: int, generator: torch.Generator | None = None
                ) -> tuple[torch.Tensor, torch.Tensor]:  # fmt: skip
    """Untrusted sampler: the k largest logits per row, then one token drawn from their
    softmax. Returns (selected (B, k), token (B,))."""
    top, idx = torch.topk(logits, k, dim=-1)
    draw = torch.multinomial(torch.softmax(top, dim=-1), 1, generator=generator)
    return idx, idx.gather(-1, draw).squeeze(-1)


def topp_select(logits: torch.Tensor, p: float, temperature: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Untrusted top-p: binary32 softmax, stable descending sort, then the shortest prefix whose
    running mass (accumulated in binary64) reaches p. Returns (order (B, V), lengths (B,));
    row b's nucleus is order[b, :lengths[b]]."""
    probs = torch.softmax(logits / temperature, dim=-1)
    sorted_probs, order = torch.sort(probs, dim=-1, descending=True, stable=True)
    running = torch.cumsum(sorted_probs.double(), dim=-1)
    lengths = ((running < p).sum(dim=-1) + 1).clamp(max=logits.shape[1])
    return order.contiguous(), lengths.to(torch.int64)


def sharded_topk_gpu(logits: torch.Tensor, k: int, shards: int, per_shard: int) -> torch.Tensor:
    """Untrusted approximate top-k (a known fault): the best ``per_shard`` of each of ``shards``
    equal slices of the vocabulary, then the best k of that pool (src/pck/faults.py:23-42)."""
    rows, vocab = logits.shape
    if vocab % shards or per_shard > vocab // shards or k > shards * per_shard:
        raise ValueError("need vocab % shards == 0, per_shard <= vocab / shards, k <= pool")
    width = vocab // shards
    _, local = torch.topk(logits.view(rows, shards, width), per_shard, dim=-1)
    pool = (local + torch.arange(shards, device=logits.device).view(1, shards, 1) * width).view(rows, -1)
    _, best = torch.topk(logits.gather(-1, pool), k, dim=-1)
    return pool.gather(-1, best)
