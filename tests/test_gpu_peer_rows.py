"""The fused all-gather on two GPUs: the FFN-down GEMM epilogue writes each
rank's rows into every rank's gathered tensor (CUDA IPC over NVLink,
parallel.PeerRows), and the gathered tensor equals the unsharded block.

Runs as two spawned NCCL ranks with a short process-group timeout; skipped
where fewer than two GPUs are visible.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from lynnreal_omni_b200 import block, _lib
    from lynnreal_omni_b200.parallel import PeerRows, shard_bounds
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    peer = None
    try:
        total, hidden = 600, 512
        w = block.make_weights(seed=0, device=dev, hidden=hidden, ffn=1024, text_dim=256)
        blk = block.FlashBlockW8A8(w)
        x, table, idx, ctx = block.make_inputs(total, seed=3, device=dev, hidden=hidden, text_tokens=64,
                                               text_dim=256)
        start, stop = shard_bounds(total, world, rank)
        peer = PeerRows(total, hidden, dev)
        results = []
        for step in range(3):  # both buffers, and one reused
            slot = step & 1
            blk(x[:, start:stop].contiguous(), table, idx[start:stop].contiguous(), ctx,
                rows_to=peer.destinations(slot))
            peer.barrier()
            full, _ = blk(x, table, idx, ctx)
            results.append(torch.equal(peer.local[slot], full.view(total, hidden)))
        torch.cuda.synchronize()
        dist.barrier()
        status = _lib.device_status(clear=True)
        queue.put((rank, all(results) and status == 0))
    except Exception as error:  # report instead of hanging the other rank
        queue.put((rank, f"{type(error).__name__}: {error}"))
    finally:
        if peer is not None:
            torch.cuda.synchronize()
            dist.barrier()
            peer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ffn_down_epilogue_gathers_rows_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert results == {0: True, 1: True}, results
