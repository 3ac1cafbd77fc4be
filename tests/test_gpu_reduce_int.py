"""Integer reductions and their elementwise neighbours on the B200, bit-exact
against the reference's outputs (golden cases), through each bundle's
candidate_kernel shim, and against the oracle on large, unaligned and
edge-case inputs (ties across blocks, all-equal arrays, chunk boundaries of
the prefix scan, both head-group reduce paths)."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from reduce_family import (RD_BUNDLES, ctypes_args, golden_case, golden_cases, library_call,
                           out_buffer)

pytestmark = pytest.mark.gpu

SHIMS = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"
RD_CASES = golden_cases(golden("reduce_family"))


@pytest.mark.parametrize("bundle,case", RD_CASES)
def test_reduce_family_golden(hx, bundle, case):
    arr = golden_case(golden("reduce_family"), bundle, case)
    np.testing.assert_array_equal(library_call(hx, bundle, arr), arr["out"])


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


@pytest.mark.parametrize("bundle", sorted(RD_BUNDLES))
def test_reduce_family_shims(hx, bundle):
    """Each bundle's candidate_kernel shim on every golden case."""
    g = golden("reduce_family")
    for b, case in RD_CASES:
        if b != bundle:
            continue
        arr = golden_case(g, bundle, case)
        out = out_buffer(bundle, arr)
        shim(bundle)(*ctypes_args(bundle, arr, out))
        np.testing.assert_array_equal(out, arr["out"], err_msg=f"{bundle} {case}")


OPS = ["sum", "sum64", "sumsq", "sumsq_diff", "dot", "l1", "absmax", "max", "min", "argmax",
       "argmin", "top1", "mean"]
DTYPES = [np.int8, np.uint8, np.int16, np.int32]


def full_range(rng, dt, n):
    info = np.iinfo(dt)
    return rng.integers(info.min, info.max + 1, n, dtype=np.int64).astype(dt)


@pytest.mark.parametrize("dt", DTYPES, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("n", [1, 15, 16, 17, 1000, (1 << 24) + 13])
def test_reduce_int_random(hx, oracle, dt, n):
    rng = np.random.default_rng(n * 7 + np.dtype(dt).itemsize)
    a, b = full_range(rng, dt, n), full_range(rng, dt, n)
    for op in OPS:
        bb = b if op in ("sumsq_diff", "dot") else None
        assert hx.reduce_int(a, op, bb) == oracle.reduce_int(a, op, bb), (op, n)


def test_reduce_int_unaligned_and_ties(hx, oracle):
    rng = np.random.default_rng(11)
    base = rng.integers(-128, 128, (1 << 22) + 40, dtype=np.int64).astype(np.int8)
    for off in (1, 3, 7):
        a, b = base[off:], base[:-off]
        for op in OPS:
            bb = b if op in ("sumsq_diff", "dot") else None
            assert hx.reduce_int(a, op, bb) == oracle.reduce_int(a, op, bb), (op, off)
    # the extreme only far apart (different blocks), all-equal, extreme last
    n = 1 << 23
    a = np.zeros(n, np.int8)
    for op in ("argmax", "argmin", "top1", "max", "min", "absmax"):
        assert hx.reduce_int(a, op) == oracle.reduce_int(a, op)
    a[[n - 1, 5_000_000, 3_000_001]] = 127
    a[[n - 2, 4_000_000]] = -128
    for op in ("argmax", "argmin", "top1", "absmax"):
        assert hx.reduce_int(a, op) == oracle.reduce_int(a, op), op
    a32 = np.full(1 << 20, -2**31, np.int32)
    for op in OPS:
        bb = a32[::-1].copy() if op in ("sumsq_diff", "dot") else None
        assert hx.reduce_int(a32, op, bb) == oracle.reduce_int(a32, op, bb), op


def test_reduce_int_empty(hx):
    e = np.zeros(0, np.int8)
    for op in ("sum", "sumsq", "l1", "max", "absmax"):
        assert hx.reduce_int(e, op) == 0
    assert hx.reduce_int(np.zeros(0, np.int32), "sum64") == 0
    for op in ("argmax", "top1", "mean"):
        with pytest.raises(RuntimeError):
            hx.reduce_int(e, op)


@pytest.mark.parametrize("dt", [np.int8, np.uint8, np.int16], ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("n", [1, 17, 4099, (1 << 22) + 5])
def test_minmax_ew_random(hx, oracle, dt, n):
    rng = np.random.default_rng(n + np.dtype(dt).itemsize)
    a, b = full_range(rng, dt, n + 1), full_range(rng, dt, n + 1)
    for op in ("max", "min"):
        np.testing.assert_array_equal(hx.minmax_ew(a[:n], b[:n], op=op), oracle.minmax_ew(a[:n], b[:n], op=op))
        np.testing.assert_array_equal(hx.minmax_ew(a[1:], b[1:], op=op), oracle.minmax_ew(a[1:], b[1:], op=op))
        for c in (-128, 0, 77):
            np.testing.assert_array_equal(hx.minmax_ew(a[:n], None, c, op), oracle.minmax_ew(a[:n], None, c, op))


def test_group_sum_and_scan(hx, oracle):
    rng = np.random.default_rng(12)
    x = rng.integers(-128, 128, (1 << 22) + 44, dtype=np.int64).astype(np.int8)
    for w in (4, 3, 1, 64):
        np.testing.assert_array_equal(hx.group_sum_i8(x, w), oracle.group_sum_i8(x, w))
    np.testing.assert_array_equal(hx.group_sum_i8(x[1:], 4), oracle.group_sum_i8(x[1:], 4))
    for n in (1, 63, 64, 16384, 3 * 16384 + 5, (1 << 24) + 7):
        v = x[:n] if n <= x.size else rng.integers(-128, 128, n, dtype=np.int64).astype(np.int8)
        np.testing.assert_array_equal(hx.scan_max_i8(v), oracle.scan_max_i8(v))
    ramp = (np.arange(200000) % 256 - 128).astype(np.int8)       # rises, resets, rises
    np.testing.assert_array_equal(hx.scan_max_i8(ramp), oracle.scan_max_i8(ramp))
    np.testing.assert_array_equal(hx.scan_max_i8(ramp[::-1].copy()), oracle.scan_max_i8(ramp[::-1].copy()))
    np.testing.assert_array_equal(hx.scan_max_i8(x[5:100005]), oracle.scan_max_i8(x[5:100005]))


@pytest.mark.parametrize("H,G,M,N", [(32, 8, 64, 64), (8, 2, 5, 33), (7, 2, 16, 16), (4, 4, 1, 1),
                                     (2, 3, 4, 4)])
def test_head_group_reduce(hx, oracle, H, G, M, N):
    rng = np.random.default_rng(H * G + M)
    X = rng.integers(-128, 128, (H, M, N), dtype=np.int64).astype(np.int8)
    for mult, shift in ((1 << 22, 24), (-123457, 9), (1, 0), (2**31 - 1, 63)):
        np.testing.assert_array_equal(hx.head_group_reduce_i8(X, G, mult, shift),
                                      oracle.head_group_reduce_i8(X, G, mult, shift))
