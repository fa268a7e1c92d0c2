"""Row-sharded checked GEMVs over the GPUs of one node (one process per GPU).

Every matrix is split by whole checker blocks: rank r owns the blocks
[r*q, min((r+1)*q, nb)) with q = ceil(nb / world), so each block's check is local to one
rank and needs nothing from the others. After the local launches, one all-gather
assembles the outputs of all projections (and the verdict bits) on every rank: NCCL's
all_gather_into_tensor, or (`Exchange.use_peer_memory`) this library's kernel that stores
each rank's slice straight into every peer's memory over NVLink (`pck_peer_all_gather`).
A rank with fewer blocks pads its slice, so every rank sends the same count.
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


class PeerTransport:
    """The all-gather of one (local, gathered) buffer pair over peer memory: an exchange
    buffer per rank from the library (`pck_peer_alloc`), mapped into every other rank with
    CUDA IPC, and one `pck_peer_all_gather` kernel per call on the current stream. Built
    collectively (every rank at the same point, like a process group call); `close()` is
    collective too."""

    def __init__(self, local: torch.Tensor, gathered: torch.Tensor, world: int, rank: int, group=None) -> None:
        import ctypes

        import torch.distributed as dist

        from pck.cuda import _lib

        if not 2 <= world <= _lib.PEER_MAX_RANKS:
            raise ValueError(f"peer memory serves 2 to {_lib.PEER_MAX_RANKS} ranks, got {world}")
        slice_bytes = local.numel() * local.element_size()
        if gathered.numel() * gathered.element_size() != world * slice_bytes or slice_bytes % 16:
            raise ValueError("gathered must hold world slices of a multiple of 16 bytes")
        self.lib, self.group, self.world, self.rank = _lib.library(), group, world, rank
        self.device = local.device
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            size = self.lib.pck_peer_buffer_bytes(slice_bytes, world)
            _lib.check(self.lib.pck_peer_alloc(size, ctypes.byref(own)), "peer buffer")
            handle = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES)()
            _lib.check(self.lib.pck_peer_export(own, handle), "peer export")
            handles: list[bytes | None] = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.own, self.mapped = own, []
            self.desc = _lib.PeerGather()
            for r in range(world):
                if r == rank:
                    self.desc.buffers[r] = own.value
                    continue
                q = ctypes.c_void_p()
                h = (ctypes.c_ubyte * _lib.PEER_HANDLE_BYTES).from_buffer_copy(handles[r])
                _lib.check(self.lib.pck_peer_import(h, ctypes.byref(q)), "peer import")
                self.mapped.append(q)
                self.desc.buffers[r] = q.value
        self.desc.local, self.desc.gathered = local.data_ptr(), gathered.data_ptr()
        self.desc.slice_bytes, self.desc.rank, self.desc.world = slice_bytes, rank, world
        self._keep = (local, gathered)

    def gather(self) -> None:
        import ctypes

        from pck.cuda import _lib
        from pck.cuda._ext import stream_handle

        rc = self.lib.pck_peer_all_gather(ctypes.byref(self.desc), stream_handle(self.device))
        _lib.check(rc, "peer all-gather")

    def close(self) -> None:
        """Unmaps the peers' buffers, waits for every rank to do the same, frees this one's."""
        import torch.distributed as dist

        from pck.cuda import _lib

        if self.own is None:
            return
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            for q in self.mapped:
                _lib.check(self.lib.pck_peer_close(q), "peer close")
            self.mapped = []
            dist.barrier(group=self.group)
            _lib.check(self.lib.pck_peer_free(self.own), "peer free")
        self.own = None


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
        self.world, self.rank = world, rank
        self.peer: PeerTransport | None = None

    def use_peer_memory(self, group=None) -> None:
        """Gathers over peer memory from now on (collective: every rank calls it)."""
        if self.peer is None:
            self.peer = PeerTransport(self.local, self.gathered, self.world, self.rank, group)

    @property
    def transport(self) -> str:
        return "peer" if self.peer is not None else "nccl"

    def gather(self, group=None) -> None:
        import torch.distributed as dist

        if self.peer is not None:
            self.peer.gather()
            return
        dist.all_gather_into_tensor(self.gathered, self.local, group=group)

    def close(self) -> None:
        """Releases the peer-memory transport (collective), if any."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None
