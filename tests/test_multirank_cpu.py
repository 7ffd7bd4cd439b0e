"""The multi-GPU host logic (sample sharding + output all-gather) on two gloo ranks, CPU only.

Each rank runs its contiguous shard of a batch through the compiled program (the noise-free
host execution stands in for the GPU evaluation: same program, same sample layout) and the
shards are reassembled with the same gather code the GPU path uses; every rank must end up
with exactly the full-batch result, including uneven shards.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN_DIR, load_package


def _worker(rank, world, port, batch, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pnb = load_package()
        with open(os.path.join(GOLDEN_DIR, "ref_phase4_cnn_fixture.json")) as f:
            d = json.load(f)
        plan = pnb.Plan(pnb.Graph(d["graph"]))
        rng = np.random.default_rng(5)
        x = rng.integers(0, 16, (batch, plan.input_elems))
        a, b = pnb.shard(batch, world, rank)
        local, _ = plan.simulate(x[a:b]) if b > a else (np.zeros((0, plan.output_elems)), 0)
        full = pnb.gather_shards(torch.tensor(local, dtype=torch.int64), batch)
        want, _ = plan.simulate(x)
        q.put((rank, bool(np.array_equal(full.numpy(), want)), (a, b)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [7, 2, 1])
def test_two_rank_shard_and_gather(batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + batch
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res)
    spans = sorted(s for _, _, s in res)
    assert spans[0][0] == 0 and spans[-1][1] == batch and spans[0][1] == spans[1][0]


def test_shard_bounds():
    pnb = load_package()
    for batch in range(0, 20):
        for world in (1, 2, 3, 8):
            spans = [pnb.shard(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_native_shard_matches_host_shard():
    # pnb_shard (the C ABI's shard rule, host-only code) agrees with the Python helper and
    # rejects out-of-range ranks.
    pnb = load_package()
    for batch in (0, 1, 7, 1024, 10**9 + 7):
        for world in (1, 2, 3, 8):
            for r in range(world):
                assert pnb.shard_native(batch, world, r) == pnb.shard(batch, world, r)
    with pytest.raises(pnb.LibraryError):
        pnb.shard_native(8, 2, 2)
    with pytest.raises(pnb.LibraryError):
        pnb.shard_native(-1, 2, 0)


def test_comm_id_is_drawn_without_a_gpu():
    # The communicator id is a host-side bootstrap address: drawing one needs no device.
    pnb = load_package()
    a, b = pnb.Comm.unique_id(), pnb.Comm.unique_id()
    assert len(a) == 128 and a != b
