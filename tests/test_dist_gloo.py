"""The N > 1 path of bench.py on CPU ranks (gloo, world size 2): the row /
M / head shards cover the problem exactly once, per-rank results assemble to
the single-process result, and the job time is the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank, world, port, out_q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    import bench
    from oracle import oracle as o

    d = bench.Dist(world)
    d.init("gloo")
    try:
        R, C = 96, 256
        rng = np.random.default_rng(0)
        x = (rng.standard_normal((R, C)) * 8).astype(np.float32)
        r0, r1 = bench.shard(R, world, rank)
        part = o.softmax(x[r0:r1])
        parts = [None] * world
        dist.all_gather_object(parts, (r0, r1, part))
        t = d.max(float(rank + 1) * 0.25)
        # heads of the attention workload and M rows of the GEMMs shard the same way
        heads = [bench.shard(256, world, r) for r in range(world)]
        if rank == 0:
            out_q.put((parts, t, heads))
        d.barrier()
    finally:
        d.close()


@pytest.mark.timeout(300)
def test_two_rank_sharding_and_max_timing():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    parts, t, heads = q.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import oracle as o
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((96, 256)) * 8).astype(np.float32)
    full = o.softmax(x)
    covered = np.zeros(96, int)
    for r0, r1, part in parts:
        np.testing.assert_array_equal(part, full[r0:r1])
        covered[r0:r1] += 1
    assert (covered == 1).all()
    assert t == 0.5
    assert heads[0] == (0, 128) and heads[1] == (128, 256)


def test_shard_covers_every_row_once():
    import bench
    for total in (1, 7, 65536, 16384, 256):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
