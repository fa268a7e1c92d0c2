"""The all-gather over peer memory (`pck_peer_all_gather`, `Exchange.use_peer_memory`)
against NCCL's all_gather_into_tensor on two GPUs: bit-identical results on every call
(both receive regions), inside a CUDA graph too, and no bounded wait giving up."""

from __future__ import annotations

import os
import socket

import pytest
import torch

CALLS = 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int) -> None:
    import datetime

    import torch.distributed as dist

    from pck.cuda import device_status
    from pck.cuda.sharded import Exchange

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)  # fmt: skip
    try:
        ms, block, batch = [4096, 1024, 14336, 640], 128, 3
        ex = Exchange([(ms, block, batch, torch.float32), ([m // block for m in ms], 1, 2, torch.bool)], world, rank, dev)
        ref = torch.empty_like(ex.gathered)
        ex.use_peer_memory()
        assert ex.transport == "peer"
        gen = torch.Generator(device=dev).manual_seed(100 + rank)
        for call in range(CALLS):
            ex.local.copy_(torch.randint(0, 256, ex.local.shape, generator=gen, device=dev, dtype=torch.uint8))
            ex.gather()
            dist.all_gather_into_tensor(ref, ex.local)
            torch.cuda.synchronize()
            assert torch.equal(ex.gathered, ref), f"rank {rank} call {call}"
        # captured: three gathers per graph, each after a local change
        src = [torch.randint(0, 256, ex.local.shape, generator=gen, device=dev, dtype=torch.uint8) for _ in range(3)]
        outs = [torch.empty_like(ex.gathered) for _ in range(3)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(3):
                ex.local.copy_(src[i])
                ex.gather()
                outs[i].copy_(ex.gathered)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        for i in range(3):
            dist.all_gather_into_tensor(ref, src[i])
            torch.cuda.synchronize()
            assert torch.equal(outs[i], ref), f"rank {rank} captured gather {i}"
        assert device_status(clear=True) == 0
        del g
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_peer_all_gather_matches_nccl_on_two_gpus() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one node")
    import torch.multiprocessing as mp

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_exchange_defaults_to_nccl_and_peer_needs_two_ranks() -> None:
    from pck.cuda.sharded import Exchange, PeerTransport

    ex = Exchange([([256], 128, 1, torch.float32)], 1, 0, "cpu")
    assert ex.transport == "nccl" and ex.peer is None
    with pytest.raises(ValueError, match="2 to 8 ranks"):
        PeerTransport(ex.local, ex.gathered, 1, 0)
