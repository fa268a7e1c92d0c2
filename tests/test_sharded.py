"""Row sharding of checked GEMVs over ranks (the multi-GPU plumbing of bench.py), on the
CPU: whole checker blocks per rank, padded equal-size chunks, and one all-gather that
reassembles every projection — run as two gloo ranks with the C oracle standing in for
the per-rank GEMV."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.gemv import gemv_coalesced_c


def test_shards_partition_rows_in_whole_blocks() -> None:
    from pck.cuda.sharded import shard_rows

    for m, block in [(4096, 128), (128256, 128), (1024, 1), (384, 128), (128, 128)]:
        for world in (1, 2, 3, 4, 8):
            shards = [shard_rows(m, block, world, r) for r in range(world)]
            assert shards[0].row0 == 0 and shards[-1].row1 == m
            for a, b in zip(shards, shards[1:]):
                assert a.row1 == b.row0
            for s in shards:
                assert s.row0 % block == 0 and s.row1 % block == 0 or s.row1 == m
                assert 0 <= s.rows <= s.rows_padded and s.rows_padded == shards[0].rows_padded
    with pytest.raises(ValueError, match="divide"):
        shard_rows(100, 128, 2, 0)
    with pytest.raises(ValueError, match="rank"):
        shard_rows(256, 128, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, batch: int, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pck.cuda.sharded import PackedOutputs, shard_rows

        block, n = 128, 256
        ms = [384, 128, 640]  # 3, 1 and 5 blocks: uneven over 2 ranks
        rng = np.random.default_rng(0)
        mats = [(rng.standard_normal((m, n)) * 0.02).astype(np.float32) for m in ms]
        xs = (rng.standard_normal((batch, n))).astype(np.float32)
        to_bits = lambda a: torch.from_numpy(a).bfloat16().view(torch.uint16).numpy()  # noqa: E731
        ys = PackedOutputs(ms, block, world, rank, "cpu", batch=batch)
        for j, W in enumerate(mats):
            sh = shard_rows(ms[j], block, world, rank)
            local = np.stack([gemv_coalesced_c(to_bits(W[sh.row0 : sh.row1]), to_bits(xs[b]), 64, 8)
                              for b in range(batch)])  # fmt: skip
            view = ys.local_view(j)
            view.copy_(torch.from_numpy(local[0] if batch == 1 else local))
        ys.gather()
        for j, W in enumerate(mats):
            full = np.stack([gemv_coalesced_c(to_bits(W), to_bits(xs[b]), 64, 8) for b in range(batch)])
            got = ys.assemble(j).numpy()
            np.testing.assert_array_equal(got.reshape(full.shape).view(np.uint32), full.view(np.uint32))
        # outputs and verdict bits in one buffer, one gather
        from pck.cuda.sharded import Exchange

        ex = Exchange([(ms, block, batch, torch.float32), ([m // block for m in ms], 1, 2, torch.bool)], world, rank,
                      "cpu")  # fmt: skip
        yv, vv = ex.parts
        for j, m in enumerate(ms):
            sh = shard_rows(m, block, world, rank)
            yv.local_view(j).copy_(torch.arange(sh.row0, sh.row1, dtype=torch.float32).expand(batch, -1).squeeze(0))
            nb0, nb1 = sh.row0 // block, sh.row1 // block
            vv.local_view(j).copy_((torch.arange(nb0, nb1) % 3 == 0).expand(2, -1))
        with pytest.raises(RuntimeError, match="Exchange"):
            yv.gather()
        ex.gather()
        for j, m in enumerate(ms):
            assert torch.equal(yv.assemble(j), torch.arange(m, dtype=torch.float32).expand(batch, -1).squeeze(0))
            assert torch.equal(vv.assemble(j), (torch.arange(m // block) % 3 == 0).expand(2, -1))
            # into fixed buffers (the LM head's captured step)
            fixed = torch.full((batch, m) if batch > 1 else (m,), -1.0)
            yv.assemble(j, out=fixed)
            assert torch.equal(fixed, torch.arange(m, dtype=torch.float32).expand(batch, -1).squeeze(0))
            bits = torch.zeros((2, m // block), dtype=torch.bool)
            vv.assemble(j, out=bits)
            assert torch.equal(bits, (torch.arange(m // block) % 3 == 0).expand(2, -1))
        out[rank] = True
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [1, 3])
def test_two_gloo_ranks_reassemble_the_full_outputs(batch: int) -> None:
    world = 2
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), batch, out), nprocs=world, join=True,
                       start_method="spawn")  # fmt: skip
    assert dict(out) == {0: True, 1: True}
