"""Token-row sharding and the output all-gather on world-size-2 gloo ranks (CPU)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lynnreal_omni_b200.parallel import frame_bounds, gather_rows, shard_bounds, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_rows_exactly():
    for total in (0, 1, 7, 1530, 12240, 64512):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_frame_bounds_are_whole_frames():
    for frames, world in ((21, 8), (21, 2), (5, 4), (3, 3)):
        spans = [frame_bounds(frames, 3072, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == frames * 3072
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all(s % 3072 == 0 and e % 3072 == 0 for s, e in spans)


def _worker(rank, world, port, total, queue, frames=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        full = torch.arange(total * 6, dtype=torch.float32).view(1, total, 6)
        bounds = None
        if frames:  # uneven whole-frame shards (token compression)
            bounds = [frame_bounds(frames, total // frames, world, r) for r in range(world)]
            local = full[:, bounds[rank][0]:bounds[rank][1]]
        else:
            local = shard_rows(full, world, rank)
        # stand-in for the per-rank W8A8 path: any row-local function
        out_local = (local * 2 + 1).view(-1, 6)
        gathered = gather_rows(out_local, total, bounds=bounds)
        queue.put((rank, torch.equal(gathered, (full * 2 + 1).view(total, 6))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total,frames", [(8, 0), (13, 0), (15, 5)])
def test_gather_rows_world2_gloo(total, frames):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, total, queue, frames)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def _dying_worker(rank, world, port, queue):
    """Rank 1 leaves before the collective; rank 0's collective must end with an
    error within the process-group timeout instead of waiting forever."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        queue.put((1, "left"))
        queue.close()
        queue.join_thread()  # flush before leaving without cleanup
        os._exit(0)
    try:
        gather_rows(torch.zeros(4, 6), 8)
        queue.put((0, "completed"))
    except Exception as error:  # gloo raises on timeout / connection loss
        queue.put((0, type(error).__name__))


def test_rank_failure_surfaces_as_error():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    assert results[0] != "completed"
