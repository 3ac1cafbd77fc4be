"""The no-allocation u8 x s8 GEMM entry (hexcuda_gemm_u8s8_pc_noalloc).

Some callers cannot let the library allocate device memory: a serving
runtime that reserved the GPU's memory for its own arena (a library
cudaMalloc would fail there), or a latency-bound caller that cannot take the
implicit synchronisation of cudaMalloc.  This entry keeps its scratch in a
fixed region compiled into libhexcuda.  Its output must equal the regular
entry's and the oracle's (integer arithmetic: bit for bit) on calls in a row
-- a later call with a smaller N or K than an earlier one would show column
sums or K padding left over from that call -- and it must reject shapes
beyond its fixed limits with the matching message.

The file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(rng, M, N, K):
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = rng.integers(36, 44, N).astype(np.int32)
    return A, B, bias, mult, shift


def _run(lib, fn, A, B, bias, mult, shift, zpa, zp_out):
    import torch
    M, K = A.shape
    N = B.shape[1]
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dbias = torch.from_numpy(bias).cuda()
    dm = torch.from_numpy(mult).cuda()
    ds = torch.from_numpy(shift).cuda()
    out = torch.full((M, N), 0xA5, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    rc = fn(0, dA.data_ptr(), dB.data_ptr(), dbias.data_ptr(), out.data_ptr(), M, N, K, zpa,
            dm.data_ptr(), ds.data_ptr(), zp_out)
    assert rc == 0, lib.hexcuda_last_error_string()
    assert lib.hexcuda_sync(0) == 0, lib.hexcuda_last_error_string()
    return out.cpu().numpy()


# (M, N, K, zpA): the 256-wide and 128-wide tile paths, with and without the
# zero-point term, a K that needs zero padding to the 128-byte K step (144),
# and a larger call followed by smaller ones
CASES = [(1000, 768, 1024, 128), (333, 1200, 640, -5), (200, 96, 256, 0), (150, 128, 144, 77),
         (64, 1000, 144, 0), (517, 64, 512, -128)]


def test_noalloc_matches_regular_entry_and_oracle_on_calls_in_a_row(hx, oracle):
    from hexkernels_b200 import _lib
    lib = _lib.load()
    lib.hexcuda_reset_stream(0)
    rng = np.random.default_rng(2024)
    for (M, N, K, zpa) in CASES:
        A, B, bias, mult, shift = _case(rng, M, N, K)
        ref = _run(lib, lib.hexcuda_gemm_u8s8_pc, A, B, bias, mult, shift, zpa, 128)
        got = _run(lib, lib.hexcuda_gemm_u8s8_pc_noalloc, A, B, bias, mult, shift, zpa, 128)
        np.testing.assert_array_equal(got, ref, err_msg=str((M, N, K, zpa)))
        np.testing.assert_array_equal(got, oracle.gemm_u8s8_pc(A, B, bias, zpa, mult, shift, 128),
                                      err_msg=str((M, N, K, zpa)))
        assert 10 < got.std()


def test_noalloc_at_the_fixed_limit(hx, oracle):
    """round_up(K, 128) * N equal to the 16 MiB region, N at its maximum."""
    from hexkernels_b200 import _lib
    lib = _lib.load()
    lib.hexcuda_reset_stream(0)
    rng = np.random.default_rng(7)
    M, N, K = 40, 16384, 1024
    A, B, bias, mult, shift = _case(rng, M, N, K)
    got = _run(lib, lib.hexcuda_gemm_u8s8_pc_noalloc, A, B, bias, mult, shift, 128, 128)
    np.testing.assert_array_equal(got, oracle.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128))


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch(hx):
    from hexkernels_b200 import _lib
    lib = _lib.load()
    out = np.zeros(4, np.uint8)
    fn = lib.hexcuda_gemm_u8s8_pc_noalloc
    # rejected before any pointer is dereferenced; each message names the
    # limit that refused it
    p = out.ctypes.data
    for (N, K, msg) in [(20000, 128, b"fixed scratch"),      # N above the column-sum region
                        (8192, 4096, b"fixed scratch"),      # K * N above the B region
                        (16384, 1040, b"fixed scratch"),     # round_up(K, 128) = 1152: one step over
                        (256, 100, b"16-byte aligned")]:     # K not a multiple of 16
        assert fn(0, p, p, p, p, 8, N, K, 128, p, p, 128) == 1, (N, K)
        assert msg in lib.hexcuda_last_error_string(), (N, K, lib.hexcuda_last_error_string())
