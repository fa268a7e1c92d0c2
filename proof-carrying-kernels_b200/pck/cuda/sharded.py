"""Row-sharded checked GEMVs over the GPUs of one node (one process per GPU).

Every matrix is split by whole checker blocks: rank r owns the blocks
[r*q, min((r+1)*q, nb)) with q = ceil(nb / world), so each block's check is local to one
rank and needs nothing from the others. After the local launches, one NCCL
all_gather_into_tensor assembles the outputs of all projections (and one the verdict
bits) on every rank; a rank with fewer blocks pads its slice, so every rank sends the
same count.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class RowShard:
    """Rows [row0, row1) of an (m, n) matrix owned by one rank, and the padded row count
    every rank contributes to the gather (``rows_padded``)."""

    row0: int
    row1: int
    rows_padded: int

    @property
    def rows(self) -> int:
        return self.row1 - self.row0


def shard_rows(m: int, block: int, world: int, rank: int) -> RowShard:
    if block < 1 or m % block:
        raise ValueError(f"block={block} must divide m={m}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    nb = m // block
    q = -(-nb // world)
    b0 = min(rank * q, nb)
    b1 = min(b0 + q, nb)
    return RowShard(b0 * block, b1 * block, q * block)


class PackedOutputs:
    """Local outputs of several sharded projections packed in one buffer per rank, so one
    all-gather moves them all. Projection j occupies a chunk of batch * rows_padded values;
    its local output is the leading (batch, rows) of that chunk (contiguous). With
    ``buffers`` (from an Exchange) the values live in a section of shared byte buffers."""

    def __init__(self, ms: Sequence[int], block: int, world: int, rank: int,
                 device: torch.device | str, batch: int = 1, dtype: torch.dtype = torch.float32,
                 buffers: tuple[torch.Tensor, torch.Tensor, int, int] | None = None) -> None:  # fmt: skip
        self.ms, self.block, self.world, self.rank, self.batch = list(ms), block, world, rank, batch
        self.dtype = dtype
        self.padded = [shard_rows(m, block, world, 0).rows_padded for m in self.ms]
        self.offsets = []
        off = 0
        for p in self.padded:
            self.offsets.append(off)
            off += batch * p
        self.per_rank = off
        self._section = buffers is not None
        if buffers is None:
            self.local = torch.zeros(off, dtype=dtype, device=device)
            self.gathered = torch.zeros(world * off, dtype=dtype, device=device)
            self._ranks = [self.gathered[r * off : (r + 1) * off] for r in range(world)]
        else:
            local, gathered, start, stride = buffers
            size = off * dtype.itemsize
            self.local = local[start : start + size].view(dtype)
            self.gathered = gathered
            self._ranks = [gathered[r * stride + start : r * stride + start + size].view(dtype)
                           for r in range(world)]  # fmt: skip

    @staticmethod
    def nbytes(ms: Sequence[int], block: int, world: int, batch: int, dtype: torch.dtype) -> int:
        return batch * sum(shard_rows(m, block, world, 0).rows_padded for m in ms) * dtype.itemsize

    def _chunk(self, buf: torch.Tensor, j: int, r: int) -> torch.Tensor:
        rows = shard_rows(self.ms[j], self.block, self.world, r).rows
        start = self.offsets[j]
        flat = buf[start : start + self.batch * rows]
        return flat if self.batch == 1 else flat.view(self.batch, rows)

    def local_view(self, j: int) -> torch.Tensor:
        """Where projection j's local outputs go: (rows,) for batch 1, else (batch, rows)."""
        return self._chunk(self.local, j, self.rank)

    def gather(self, group=None) -> None:
        import torch.distributed as dist

        if self._section:
            raise RuntimeError("a section of an Exchange is gathered by the Exchange")
        dist.all_gather_into_tensor(self.gathered, self.local, group=group)

    def assemble(self, j: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Projection j's full output, (m,) or (batch, m), from the gathered buffer (one
        concatenation kernel; into ``out`` when given, e.g. a fixed buffer of a captured step)."""
        chunks = [self._chunk(self._ranks[r], j, r) for r in range(self.world)]
        if out is None:
            return torch.cat(chunks, dim=-1)
        return torch.cat(chunks, dim=-1, out=out)


class Exchange:
    """Several PackedOutputs (e.g. a layer's outputs and its verdict bits) in one byte buffer
    per rank, each section 16-byte aligned, so a single all-gather per step moves them all.
    ``sections``: (ms, block, batch, dtype) per PackedOutputs, in `parts`."""

    def __init__(self, sections: Sequence[tuple[Sequence[int], int, int, torch.dtype]], world: int, rank: int,
                 device: torch.device | str) -> None:  # fmt: skip
        starts, off = [], 0
        for ms, block, batch, dtype in sections:
            starts.append(off)
            off += -(-PackedOutputs.nbytes(ms, block, world, batch, dtype) // 16) * 16
        self.per_rank = off
        self.local = torch.zeros(off, dtype=torch.uint8, device=device)
        self.gathered = torch.zeros(world * off, dtype=torch.uint8, device=device)
        self.parts = [PackedOutputs(ms, block, world, rank, device, batch, dtype,
                                    buffers=(self.local, self.gathered, start, off))
                      for (ms, block, batch, dtype), start in zip(sections, starts, strict=True)]  # fmt: skip

    def gather(self, group=None) -> None:
        import torch.distributed as dist

        dist.all_gather_into_tensor(self.gathered, self.local, group=group)
