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


def gather_rank_main(rank, world, port, out_q):
    """One CPU rank: computes its part of the rows with the oracle, then
    assembles the whole output with the gather plan libhexcuda's NCCL path
    follows (hexcuda_shard_rows for the parts; one all-gather when the parts
    are equal, one broadcast per owning part otherwise), over gloo."""
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist

    from hexkernels_b200 import ops
    from oracle import oracle as o

    dist.init_process_group("gloo", world_size=world, rank=rank)
    try:
        results = {}
        for R in (96, 97, 1):
            C_ = 256
            rng = np.random.default_rng(R)
            x = (rng.standard_normal((R, C_)) * 8).astype(np.float32)
            A = rng.integers(0, 256, (R, 64), dtype=np.uint8)
            B = rng.integers(-128, 128, (64, 48), dtype=np.int8)
            bias = rng.integers(-3000, 3000, 48).astype(np.int32)
            mult = rng.integers(2**30, 2**31, 48, dtype=np.int64).astype(np.int32)
            shift = np.full(48, 20, np.int32)
            spans = [ops.shard_rows(R, world, r) for r in range(world)]
            r0, r1 = spans[rank]
            outs = []
            for part, row_shape, dt in (
                    (o.softmax(x[r0:r1]), (C_,), np.float32),
                    (o.gemm_u8s8_pc(A[r0:r1], B, bias, 128, mult, shift, 128), (48,), np.uint8)):
                full = torch.zeros((R, *row_shape), dtype=torch.from_numpy(np.zeros(1, dt)).dtype)
                mine = torch.from_numpy(np.ascontiguousarray(part))
                counts = [b - a for a, b in spans]
                if all(c == counts[0] for c in counts):
                    chunks = list(torch.split(full, counts[0]))
                    dist.all_gather(chunks, mine)
                    full = torch.cat(chunks)
                else:
                    for root, (a, b) in enumerate(spans):
                        if b == a:
                            continue
                        buf = mine.clone() if root == rank else torch.empty((b - a, *row_shape),
                                                                            dtype=full.dtype)
                        dist.broadcast(buf, root)
                        full[a:b] = buf
                outs.append(full.numpy())
            results[R] = outs
        if rank == 0:
            out_q.put(results)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_replicated_output_assembles_like_one_process():
    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=gather_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = q.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from oracle import oracle as o
    for R, (sm, gm) in results.items():
        rng = np.random.default_rng(R)
        x = (rng.standard_normal((R, 256)) * 8).astype(np.float32)
        A = rng.integers(0, 256, (R, 64), dtype=np.uint8)
        B = rng.integers(-128, 128, (64, 48), dtype=np.int8)
        bias = rng.integers(-3000, 3000, 48).astype(np.int32)
        mult = rng.integers(2**30, 2**31, 48, dtype=np.int64).astype(np.int32)
        shift = np.full(48, 20, np.int32)
        np.testing.assert_array_equal(sm, o.softmax(x))
        np.testing.assert_array_equal(gm, o.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128))


def test_shard_rows_matches_bench_split():
    import bench
    from hexkernels_b200 import ops
    for total in (0, 1, 7, 97, 16384):
        for world in (1, 2, 3, 8):
            for r in range(world):
                assert ops.shard_rows(total, world, r) == bench.shard(total, world, r)
