"""Integer affine elementwise requant (hexcuda_affine_ew) on the B200,
bit-exact against the reference's outputs (golden affine: rescale_i16_i8_dma,
dequant_i8_i16_dma, hmx_requant_store_i8, i8_add_bias_sat_dma,
i8_element_affine_dma, u8_max_dma, u8_min_dma), through each bundle's
candidate_kernel shim, and against the oracle for every input / output type,
both roundings and both arithmetic widths on lengths off the vector width."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from test_oracle_golden import affine_calls

pytestmark = pytest.mark.gpu

SHIMS = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def test_affine_golden(hx):
    for k, (got, exp) in enumerate(affine_calls(hx, golden("affine"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def test_affine_shims(hx):
    g = golden("affine")
    x8, n = g["x8"], g["x8"].size
    out = np.zeros(n, np.int8)
    shim("rescale_i16_i8_dma")(p(g["rescale_i16_i8_dma__a0"]), p(out), n)
    np.testing.assert_array_equal(out, g["rescale_i16_i8_dma__out0"])
    fn = shim("dequant_i8_i16_dma")
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int8, C.c_int32, C.c_int]
    for t, (zp, scale, shift) in enumerate(((0, 1, 0), (-7, 300, 3), (100, -77777, 11), (-128, 2**22, 31))):
        o16 = np.zeros(n, np.int16)
        fn(p(x8), p(o16), n, zp, scale, shift)
        np.testing.assert_array_equal(o16, g[f"dequant_i8_i16_dma__out{t}"])
    shim("hmx_requant_store_i8")(p(g["hmx_requant_store_i8__a0"]), p(out), n)
    np.testing.assert_array_equal(out, g["hmx_requant_store_i8__out0"])
    fn = shim("i8_add_bias_sat_dma")
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int32]
    for t, bias in enumerate((0, 77, -200, 100000)):
        fn(p(x8), p(out), n, bias)
        np.testing.assert_array_equal(out, g[f"i8_add_bias_sat_dma__out{t}"])
    fn = shim("i8_element_affine_dma")
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int32, C.c_int32, C.c_int]
    for t, (scale, sh, s) in enumerate(((1, 0, 0), (3, 5, 2), (-1000, 333, 9), (2**31 - 1, -(2**31), 40))):
        fn(p(x8), p(out), n, scale, sh, s)
        np.testing.assert_array_equal(out, g[f"i8_element_affine_dma__out{t}"])
    u8 = g["u8"]
    for name in ("u8_max_dma", "u8_min_dma"):
        for t, m in enumerate((n, 1, 0)):
            o = np.zeros(1, np.uint8)
            shim(name)(p(u8), m, p(o))
            np.testing.assert_array_equal(o, g[f"{name}__out{t}"], err_msg=f"{name} {m}")


IN = [np.int8, np.uint8, np.int16, np.int32]
OUT = [np.int8, np.uint8, np.int16, np.int32]


@pytest.mark.parametrize("ti", IN, ids=lambda d: np.dtype(d).name)
@pytest.mark.parametrize("to", OUT, ids=lambda d: np.dtype(d).name)
def test_affine_random(hx, oracle, ti, to):
    rng = np.random.default_rng(np.dtype(ti).itemsize * 10 + np.dtype(to).itemsize)
    info = np.iinfo(ti)
    x = rng.integers(info.min, info.max + 1, (1 << 20) + 13, dtype=np.int64).astype(ti)
    cases = [dict(mult=3, shift=4, wrap32=True), dict(zp_in=-7, mult=300, shift=3, round="floor", wrap32=True),
             dict(mult=17, add=8, shift=4, round="floor", wrap32=True),
             dict(mult=-1000, add=333, shift=9), dict(mult=2**31 - 1, add=-(2**40), shift=50, zp_out=5),
             dict(mult=1, add=100000, round="floor", wrap32=True, lo=-50, hi=60)]
    for kw in cases:
        for xs in (x, x[1:]):
            np.testing.assert_array_equal(hx.affine_ew(xs, to, **kw), oracle.affine_ew(xs, to, **kw),
                                          err_msg=str(kw))


def test_affine_rejects_bad_arguments(hx):
    x = np.zeros(16, np.int8)
    for kw in (dict(shift=32, wrap32=True), dict(shift=63), dict(round="floor", lo=5, hi=4)):
        with pytest.raises(RuntimeError):
            hx.affine_ew(x, np.int8, **kw)


from test_oracle_golden import RELU6_SCALES, clamp_calls  # noqa: E402


def test_clamp_and_pool_golden_and_shims(hx):
    g = golden("affine")
    for k, (got, exp) in enumerate(clamp_calls(hx, g)):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))
    x8, u8, n = g["x8"], g["u8"], g["x8"].size
    for name in ("i8_relu_dma", "i8_relu_stream_dma"):
        out = np.zeros(n, np.int8)
        shim(name)(p(x8), p(out), n)
        np.testing.assert_array_equal(out, g[name + "__out0"])
    fn = shim("i8_relu6_dma")
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int8]
    for t, scale in enumerate(RELU6_SCALES):
        out = np.zeros(n, np.int8)
        fn(p(x8), p(out), n, scale)
        np.testing.assert_array_equal(out, g[f"i8_relu6_dma__out{t}"], err_msg=str(scale))
    for name in ("u8_clamp_range_dma", "dma_double_buffer_relu_u8"):
        out = np.zeros(n, np.uint8)
        shim(name)(p(u8), p(out), n)
        np.testing.assert_array_equal(out, g[name + "__out0"])
    for t, m in enumerate((n, 1, 77)):
        for name, src, dt in (("i8_global_avgpool_dma", x8, np.int8), ("u8_global_avgpool_dma", u8, np.uint8),
                              ("i8_global_maxpool_dma", x8, np.int8)):
            o = np.zeros(1, dt)
            shim(name)(p(src), m, p(o))
            np.testing.assert_array_equal(o, g[f"{name}__out{t}"], err_msg=f"{name} {m}")
    o = np.zeros(1, np.int8)
    shim("i8_global_maxpool_dma")(p(x8), 0, p(o))
    np.testing.assert_array_equal(o, g["i8_global_maxpool_dma__out3"])


def test_ew_shims(hx):
    g = golden("affine")
    x8, y8, u8, n = g["x8"], g["y8"], g["u8"], g["x8"].size
    out = np.zeros(n, np.uint8)
    shim("u8_threshold_dma")(p(u8), p(out), n)
    np.testing.assert_array_equal(out, g["u8_threshold_dma__out0"])
    out = np.zeros(n, np.int8)
    shim("i8_sign_dma")(p(x8), p(out), n)
    np.testing.assert_array_equal(out, g["i8_sign_dma__out0"])
    for name in ("i8_add_dma", "i8_add_stream_dma", "i8_vadd_dma"):
        out = np.zeros(n, np.int8)
        shim(name)(p(x8), p(y8), p(out), n)
        np.testing.assert_array_equal(out, g[name + "__out0"], err_msg=name)
