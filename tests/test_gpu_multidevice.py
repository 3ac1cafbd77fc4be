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
