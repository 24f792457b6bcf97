"""Host logic of the steering sweep: the pair plan, the sharding across ranks and
the final gather, the last on a two-rank gloo group over 127.0.0.1 (no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from frizzle_b200 import sweep


def test_pairs_are_seeded_and_in_range():
    a, b = sweep.make_pairs(64, 6912, seed=0), sweep.make_pairs(64, 6912, seed=0)
    assert len(a) == 64
    for p, q in zip(a, b):
        assert p.seed == q.seed and np.array_equal(p.neurons, q.neurons) and np.array_equal(p.values, q.values)
        assert 1 <= len(p.neurons) <= 8 and len(set(p.neurons.tolist())) == len(p.neurons)
        assert p.neurons.max() < 6912 and np.all(np.abs(p.values) <= 10.0)
        assert all(0 <= s < 2**32 for s in p.seed)
    assert sweep.make_pairs(64, 6912, seed=1)[0].seed != a[0].seed


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (7, 3), (3, 8), (0, 4)])
def test_shards_cover_once(n, world):
    seen = []
    sizes = []
    for r in range(world):
        s = sweep.shard(n, world, r)
        seen.extend(s)
        sizes.append(len(s))
    assert seen == list(range(n))
    assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, n_pairs, steps, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = sweep.shard(n_pairs, world, rank)
        results = {i: np.full((2, steps), 1000 * i + rank, dtype=np.int32) for i in mine}
        for i in mine:
            results[i][1] += 1
        full = sweep.gather(results, n_pairs, steps, dist)
        q.put((rank, None if full is None else full.tolist()))
    finally:
        dist.destroy_process_group()


def test_gather_two_ranks_gloo():
    n_pairs, steps, world = 5, 3, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, n_pairs, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[1] is None
    full = np.array(got[0])
    for i in range(n_pairs):
        owner = 0 if i in sweep.shard(n_pairs, world, 0) else 1
        assert np.all(full[i, 0] == 1000 * i + owner) and np.all(full[i, 1] == 1000 * i + owner + 1)
