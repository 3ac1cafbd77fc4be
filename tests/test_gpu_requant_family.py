"""Elementwise requant family on the B200 (HBM-streaming kernel), bit-exact
against the reference's outputs (golden cases) and the oracle (large and
unaligned cases), through the host API and through each bundle's
candidate_kernel shim."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from requant_family import RQ_BUNDLES, case_arrays, ew_kwargs
from test_oracle_golden import RQ_CASES

pytestmark = pytest.mark.gpu

SHIMS = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"


@pytest.mark.parametrize("bundle,case", RQ_CASES)
def test_requant_family_golden(hx, bundle, case):
    arr = case_arrays(golden("requant_family"), bundle, case)
    a = arr["a8"] if "a8" in arr else arr["a32"]
    np.testing.assert_array_equal(hx.requant_ew(a, **ew_kwargs(bundle, arr)), arr["out"])


def test_epilogue_bias_relu_golden(hx):
    g = golden("requant_family")
    np.testing.assert_array_equal(
        hx.epilogue_bias_i32(g["epilogue_bias_i32__acc"], g["epilogue_bias_i32__bias"]),
        g["epilogue_bias_i32__out"])
    np.testing.assert_array_equal(hx.relu_i8(g["epilogue_relu_i8__x"]), g["epilogue_relu_i8__out"])


VARIANTS = [dict(mult=1518500250, shift=38, zp=3),
            dict(pre="add", mult=-77777, shift=9, zp=-4),
            dict(pre="add_relu", mult=3, shift=4, zp=1, lo2=-20, hi2=40),
            dict(pre="mul_add", pre_c=50, mult=3, shift=21, zp=0),
            dict(mult=-1234567, shift=20, zp=7, sign_of_a=True),
            dict(mult=1 << 30, shift=40, zp=-3, lo1=0, hi1=255, lo2=0, hi2=255, lut="rand"),
            dict(mult=13, shift=3, lo1=0, hi1=24, lo2=0, hi2=24)]


@pytest.mark.parametrize("n", [1, 15, 17, 4099, (1 << 22) + 13])
@pytest.mark.parametrize("a_i8", [False, True])
def test_requant_ew_random(hx, oracle, n, a_i8):
    rng = np.random.default_rng(n + a_i8)
    if a_i8:
        a = rng.integers(-128, 128, n).astype(np.int8)
        b = rng.integers(-128, 128, n).astype(np.int8)
    else:
        a = rng.integers(-2**20, 2**20, n).astype(np.int32)
        b = rng.integers(-2**20, 2**20, n).astype(np.int32)
    lut = rng.integers(-128, 128, 256).astype(np.int8)
    for kw in VARIANTS:
        kw = dict(kw)
        if kw.get("lut") == "rand":
            kw["lut"] = lut
        bb = b if kw.get("pre", "a") != "a" else None
        np.testing.assert_array_equal(hx.requant_ew(a, bb, **kw), oracle.requant_ew(a, bb, **kw),
                                      err_msg=str(kw))


def test_requant_ew_unaligned_views(hx, oracle):
    """Inputs and output at odd byte offsets take the scalar path."""
    rng = np.random.default_rng(5)
    n = 100003
    a = rng.integers(-2**30, 2**30, n + 1).astype(np.int32)[1:]
    b = rng.integers(-2**30, 2**30, n + 3).astype(np.int32)[3:]
    kw = dict(pre="add", mult=1 << 30, shift=35, zp=2)
    np.testing.assert_array_equal(hx.requant_ew(a, b, **kw), oracle.requant_ew(a, b, **kw))
    acc = rng.integers(-2**31, 2**31, (301, 77), dtype=np.int64).astype(np.int32)
    bias = rng.integers(-2**31, 2**31, 77, dtype=np.int64).astype(np.int32)
    np.testing.assert_array_equal(hx.epilogue_bias_i32(acc, bias), oracle.epilogue_bias_i32(acc, bias))
    x = rng.integers(-128, 128, 1 << 20).astype(np.int8)
    np.testing.assert_array_equal(hx.relu_i8(x[1:]), oracle.relu_i8(x[1:]))


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


@pytest.mark.parametrize("bundle", sorted(RQ_BUNDLES))
def test_requant_shims(hx, bundle):
    """Each bundle's candidate_kernel shim on its golden cases."""
    params, _ = RQ_BUNDLES[bundle]
    for case in ("c0", "c1"):
        arr = case_arrays(golden("requant_family"), bundle, case)
        out = np.zeros_like(arr["out"])
        args = []
        for prm in params:
            if prm == "out":
                args.append(out.ctypes.data_as(C.c_void_p))
            elif prm == "n":
                args.append(C.c_int(out.size))
            elif prm == "mult":
                args.append(C.c_int32(int(arr["mult"])))
            elif prm in ("shift",):
                args.append(C.c_int(int(arr["shift"])))
            elif prm in ("zp", "lo", "hi"):
                args.append(C.c_int8(int(arr[prm])))
            else:
                args.append(arr[prm].ctypes.data_as(C.c_void_p))
        shim(bundle)(*args)
        np.testing.assert_array_equal(out, arr["out"], err_msg=f"{bundle} {case}")
