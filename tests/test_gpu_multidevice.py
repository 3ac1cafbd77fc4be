"""One process, several B200s: the host-pointer entries split rows (M rows,
B*H heads) across the initialised devices and the assembled result equals
the single-device result.  Skipped when fewer than two GPUs are visible."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hexkernels_b200 import ops
    n = ops.init(2)
    assert n == 2
    yield ops
    ops.init(1)


def test_rows_sharded_over_two_devices(two, oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((1001, 4096)) * 8).astype(np.float32)
    g = rng.normal(1, 0.1, 4096).astype(np.float32)
    b = rng.normal(0, 0.1, 4096).astype(np.float32)
    np.testing.assert_allclose(two.softmax(x), oracle.softmax(x), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(two.layernorm(x, g, b, 1e-5), oracle.layernorm(x, g, b, 1e-5),
                               rtol=1e-5, atol=1e-4)
    np.testing.assert_array_equal(two.rowreduce(x, 1), oracle.rowreduce(x, 1))


def test_gemm_sharded_over_two_devices(two, oracle):
    rng = np.random.default_rng(2)
    M, N, K = 777, 640, 1024
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = np.full(N, 38, np.int32)
    np.testing.assert_array_equal(two.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128),
                                  oracle.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128))


def test_attention_sharded_over_two_devices(two, oracle):
    rng = np.random.default_rng(3)
    Q, K, V = (rng.standard_normal((5, 300, 128)).astype(np.float16) for _ in range(3))
    got = two.attn_f16(Q, K, V, 1 / np.sqrt(128), True).astype(np.float64)
    exp = oracle.attn_f16(Q, K, V, 1 / np.sqrt(128), True).astype(np.float64)
    assert np.all(np.abs(got - exp) <= 1e-2 * np.abs(exp) + 2e-3)


def test_replicated_outputs_on_two_devices(two, oracle):
    """With replicate on, each device ends up holding the whole output (the
    other device's rows arrive by NCCL over NVLink); checked against the
    oracle on both devices, for ragged (broadcast plan) and equal (all-gather
    plan) parts."""
    two.set_replicate(True)
    try:
        rng = np.random.default_rng(4)
        x = (rng.standard_normal((1001, 4096)) * 8).astype(np.float32)   # 500 + 501 rows
        got = two.softmax(x)
        np.testing.assert_allclose(got, oracle.softmax(x), rtol=1e-5, atol=1e-7)
        for dev in (0, 1):
            np.testing.assert_array_equal(two.replica(dev, x.shape, np.float32), got)
        assert two.last_collective_ms() > 0
        M, N, K = 768, 640, 1024                                          # 384 + 384 rows
        A = rng.integers(0, 256, (M, K), dtype=np.uint8)
        B = rng.integers(-128, 128, (K, N), dtype=np.int8)
        bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
        mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
        shift = np.full(N, 38, np.int32)
        exp = oracle.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128)
        np.testing.assert_array_equal(two.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128), exp)
        for dev in (0, 1):
            np.testing.assert_array_equal(two.replica(dev, (M, N), np.uint8), exp)
        Q, Kk, V = (rng.standard_normal((6, 256, 128)).astype(np.float16) for _ in range(3))
        got = two.attn_f16(Q, Kk, V, 1 / np.sqrt(128), True)
        for dev in (0, 1):
            np.testing.assert_array_equal(two.replica(dev, Q.shape, np.float16), got)
    finally:
        two.set_replicate(False)


def test_device_pointer_allgather_two_devices(two):
    """hexcuda_allgather_rows on torch tensors of two devices, ragged rows,
    one part gathered in place."""
    import ctypes as C

    import torch

    from hexkernels_b200 import _lib
    lib = _lib.load()
    rows, width = 37, 1000
    full_ref = torch.arange(rows * width, dtype=torch.int32).reshape(rows, width)
    spans = [two.shard_rows(rows, 2, i) for i in range(2)]
    fulls = [torch.zeros((rows, width), dtype=torch.int32, device=f"cuda:{i}") for i in range(2)]
    shards = [full_ref[a:b].to(f"cuda:{i}") for i, (a, b) in enumerate(spans)]
    # device 1 gathers in place: its part already sits at its offset
    fulls[1][spans[1][0]:spans[1][1]] = shards[1]
    send = [shards[0].data_ptr(), fulls[1][spans[1][0]:].data_ptr()]
    for i in range(2):
        torch.cuda.synchronize(i)
    sp = (C.c_void_p * 2)(*send)
    fp = (C.c_void_p * 2)(*[f.data_ptr() for f in fulls])
    _lib.check(lib.hexcuda_allgather_rows(sp, fp, rows, width * 4))
    _lib.check(lib.hexcuda_sync(-1))
    for f in fulls:
        assert torch.equal(f.cpu(), full_ref)


def _rank_gather(rank, world, rows, q_id, q_out):
    import ctypes as C
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import torch

    from hexkernels_b200 import _lib, ops
    torch.cuda.set_device(rank)
    ops.init_devices([rank])
    lib = _lib.load()
    uid = C.create_string_buffer(128)
    if rank == 0:
        _lib.check(lib.hexcuda_comm_unique_id(uid, 128))
        for _ in range(world - 1):
            q_id.put(uid.raw)
    else:
        C.memmove(uid, q_id.get(timeout=120), 128)
    _lib.check(lib.hexcuda_comm_init_rank(world, rank, uid, 128))
    width = 333
    full_ref = (torch.arange(rows * width, dtype=torch.int64) % 251).to(torch.uint8).reshape(rows, width)
    a, b = ops.shard_rows(rows, world, rank)
    shard = full_ref[a:b].cuda()
    full = torch.zeros((rows, width), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    _lib.check(lib.hexcuda_comm_allgather_rows(shard.data_ptr(), full.data_ptr(), rows, width))
    _lib.check(lib.hexcuda_sync(0))
    q_out.put((rank, bool(torch.equal(full.cpu(), full_ref)), lib.hexcuda_last_collective_ms()))
    lib.hexcuda_comm_destroy()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("rows", [64, 7])
def test_multiprocess_allgather_two_ranks(rows):
    """One process per GPU (the bench's torchrun layout): hexcuda_comm_* over
    two ranks gathers equal (64 rows) and ragged (7 rows) parts."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_gather, args=(r, 2, rows, q_id, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q_out.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [True, True]
    assert all(r[2] > 0 for r in res)
