"""The library's own output all-gather (``pnb_allgather`` over NCCL) for sample-sharded
evaluation: one rank on one GPU (the collective degenerates to a copy), and, where the machine
has two or more GPUs, one process per GPU with equal and ragged shards.  Every rank must hold
exactly the rows every other rank produced."""
from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

from conftest import load_package

pytestmark = pytest.mark.gpu


def _rows(batch: int, row: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-2**62, 2**62, (batch, row), generator=g, dtype=torch.int64)


def test_single_rank_allgather_is_a_copy():
    pnb = load_package()
    uid = pnb.Comm.unique_id()
    with pnb.Comm(0, 1, 0, uid) as comm:
        x = _rows(5, 2049, 1).cuda()
        y = comm.allgather(x, 5)
        torch.cuda.synchronize()
        assert torch.equal(y, x)
        comm.status()
        with pytest.raises(ValueError):
            comm.allgather(x[:4], 5)  # a shard of the wrong size is refused on the host


def _worker(rank, world, uid, cases, q):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        pnb = load_package()
        torch.cuda.set_device(rank)
        comm = pnb.Comm(rank, world, rank, uid)
        ok = []
        for batch, row, seed in cases:
            full = _rows(batch, row, seed)
            a, b = pnb.shard(batch, world, rank)
            local = full[a:b].cuda()
            got = comm.allgather(local, batch)
            torch.cuda.synchronize()
            ok.append(bool(torch.equal(got.cpu(), full)))
        comm.status()
        comm.close()
        q.put((rank, ok, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, [], repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_multi_gpu_allgather_equal_and_ragged_shards():
    pnb = load_package()
    world = min(torch.cuda.device_count(), 4)
    uid = pnb.Comm.unique_id()
    # equal shards (one ncclAllGather), ragged shards (grouped broadcasts), fewer rows than ranks
    cases = [(8 * world, 2049, 1), (8 * world + 3, 2049, 2), (world - 1, 2050, 3), (1, 7, 4)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert ok == [True] * len(cases), f"rank {rank}: {ok}"
