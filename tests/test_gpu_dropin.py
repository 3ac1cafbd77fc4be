"""Drop-in boundary on the B200: the corpus's own harness.c programs, linked
unchanged against the candidate_kernel shims (built from the reference tree
into oracle/_ref/ by `make -C oracle ref-gpu`), print HVXENV_CORRECT; and the
new task headers' shims compute the same as the oracle when called through
candidate_kernel itself."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
REF = REPO / "oracle" / "_ref"
SHIMS = REPO / "hexkernels_b200" / "shims"

pytestmark = pytest.mark.gpu

HARNESSES = sorted(REF.glob("gpu_harness_*")) if REF.exists() else []


@pytest.mark.skipif(not HARNESSES, reason="reference harnesses not built here (make -C oracle ref-gpu)")
@pytest.mark.parametrize("exe", HARNESSES, ids=lambda p: p.name[len("gpu_harness_"):])
def test_reference_harness_links_and_passes(hx, exe):
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert "HEXCUDA_ERROR" not in r.stderr, r.stderr
    assert re.search(r"^HVXENV_CORRECT errors=0", r.stdout, re.M), r.stdout + r.stderr
    assert "HEXCUDA_KERNEL_US" in r.stdout
    assert r.returncode == 0


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    lib = C.CDLL(str(so))
    lib.candidate_kernel.restype = None
    return lib.candidate_kernel


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def test_shim_softmax_layernorm_rowreduce_f32(hx, oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 4096)) * 8).astype(np.float32)
    g = rng.normal(1, 0.1, 4096).astype(np.float32)
    b = rng.normal(0, 0.1, 4096).astype(np.float32)
    out = np.zeros_like(x)
    shim("softmax_f32")(p(x), p(out), 64, 4096)
    np.testing.assert_allclose(out, oracle.softmax(x), rtol=1e-5, atol=1e-7)
    fn = shim("layernorm_f32")
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_int, C.c_float]
    fn(p(x), p(g), p(b), p(out), 64, 4096, 1e-5)
    np.testing.assert_allclose(out, oracle.layernorm(x, g, b, 1e-5), rtol=1e-5, atol=1e-4)
    red = np.zeros(64, np.float32)
    shim("rowreduce_f32")(p(x), p(red), 64, 4096, 1)
    np.testing.assert_array_equal(red, oracle.rowreduce(x, 1))


def test_shim_gemm_u8s8_pc(hx, oracle):
    rng = np.random.default_rng(2)
    M, N, K = 300, 200, 640
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = np.full(N, 38, np.int32)
    out = np.zeros((M, N), np.uint8)
    fn = shim("gemm_u8s8_pc")
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int] * 3 + [C.c_int32, C.c_void_p, C.c_void_p, C.c_uint8]
    fn(p(A), p(B), p(bias), p(out), M, N, K, 128, p(mult), p(shift), 128)
    np.testing.assert_array_equal(out, oracle.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128))


def test_shim_attn_f16(hx, oracle):
    rng = np.random.default_rng(3)
    Bn, H, S, D = 2, 3, 200, 128
    Q, K, V = (rng.standard_normal((Bn, H, S, D)).astype(np.float16) for _ in range(3))
    O = np.zeros_like(Q)
    fn = shim("attn_f16")
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float, C.c_int]
    fn(p(Q), p(K), p(V), p(O), Bn, H, S, D, 1 / np.sqrt(D), 1)
    exp = oracle.attn_f16(Q, K, V, 1 / np.sqrt(D), True)
    assert np.all(np.abs(O.astype(np.float64) - exp) <= 1e-2 * np.abs(exp.astype(np.float64)) + 2e-3)


def test_shim_hmx_bundles(hx, oracle):
    """The six HMX-convention shims through candidate_kernel at a size that
    spans several tiles (n = 200, full-range values)."""
    rng = np.random.default_rng(3)
    n, K = 200, 520
    A = rng.integers(0, 256, (n, n), dtype=np.uint8)
    B = rng.integers(-128, 128, (n, n), dtype=np.int8)
    bias = rng.integers(-2000, 2000, n).astype(np.int32)
    o32 = np.zeros((n, n), np.int32)
    shim("hmx_matmul_i8_64")(p(A), p(B), p(o32), n)
    np.testing.assert_array_equal(o32, oracle.gemm_hmx(A, B, 0))
    shim("hmx_matmul_i8_zp")(p(A), p(B), 77, p(o32), n)
    np.testing.assert_array_equal(o32, oracle.gemm_hmx(A, B, 0, None, 77))
    Bt = np.ascontiguousarray(B.T)
    shim("hmx_matmul_i8_transposeB")(p(A), p(Bt), p(o32), n)
    np.testing.assert_array_equal(o32, oracle.gemm_hmx(A, B, 0))
    o8 = np.zeros((n, n), np.int8)
    shim("hmx_matmul_i8_requant")(p(A), p(B), p(o8), n)
    np.testing.assert_array_equal(o8, oracle.gemm_hmx(A, B, 1))
    u8 = np.zeros((n, n), np.uint8)
    shim("i8_gemm_bias_relu_requant_hmx")(p(A), p(B), p(bias), p(u8), n)
    np.testing.assert_array_equal(u8, oracle.gemm_hmx(A, B, 2, bias))
    Ad = rng.integers(0, 256, (n, K), dtype=np.uint8)
    Bd = rng.integers(-128, 128, (K, n), dtype=np.int8)
    shim("hmx_matmul_i8_deepk")(p(Ad), p(Bd), p(o32), n, K)
    np.testing.assert_array_equal(o32, oracle.gemm_hmx(Ad, Bd, 0))


@pytest.mark.parametrize("bundle", sorted(__import__("hmx_family").BUNDLES))
def test_shim_hmx_family(hx, bundle):
    """Each HMX-family shim through candidate_kernel on its golden case."""
    from conftest import golden
    from hmx_family import BUNDLES
    g = golden("hmx_family")
    params, kw = BUNDLES[bundle]
    arr = {k.split("__", 1)[1]: g[k] for k in g if k.startswith(bundle + "__")}
    M, N, K = (int(v) for v in arr["mnk"])
    out = np.zeros_like(arr["out"])
    args = []
    for prm in params:
        if prm == "out":
            args.append(p(out))
        elif prm in ("n", "M"):
            args.append(M)
        elif prm == "N":
            args.append(N)
        elif prm == "K":
            args.append(K)
        else:
            args.append(p(np.ascontiguousarray(arr[prm])))
    shim(bundle)(*args)
    np.testing.assert_array_equal(out, arr["out"])


def test_shim_int8_attention_hmx(hx):
    from conftest import golden
    g = golden("int8_attention_hmx")
    S, D = (int(v) for v in g["qkt_SD"])
    o16 = np.zeros(S * S, np.uint16)
    shim("i8_attention_qkt_hmx")(p(g["qkt_Q"]), p(g["qkt_K"]), p(o16), S, D)
    np.testing.assert_array_equal(o16, g["qkt_out"])
    o16 = np.zeros(S * D, np.uint16)
    shim("i8_attention_av_hmx")(p(g["av_P"]), p(g["av_V"]), p(o16), S, D)
    np.testing.assert_array_equal(o16, g["av_out"])
    S, D = (int(v) for v in g["qkav_SD"])
    o32 = np.zeros(S * D, np.int32)
    shim("i8_attention_qkt_av_hmx")(p(g["qkav_Q"]), p(g["qkav_K"]), p(g["qkav_V"]), p(o32), S, D)
    np.testing.assert_array_equal(o32, g["qkav_out"])
    og = np.zeros(2 * 64 * 64, np.uint16)
    shim("i8_gqa_qkt_hmx")(p(g["gqa_Q"]), p(g["gqa_K"]), p(og))
    np.testing.assert_array_equal(og, g["gqa_out"])


def test_shim_f16_family(hx):
    """The fp16 post-op shims through candidate_kernel on their golden cases
    (fp16 GEMM tolerance; hmx_tile_mac accumulates into its output)."""
    from conftest import golden
    from test_gpu_gemm import assert_f16_gemm_close
    g = golden("f16_family")
    arr = lambda b, k: np.ascontiguousarray(g[f"{b}__{k}"])
    for b in ("fp16_matmul_gelu_hmx", "fp16_matmul_hmx_32x32", "hmx_matmul_fp16_32",
              "hmx_matmul_fp16_relu", "hmx_conv1x1_fp16"):
        o = np.zeros_like(arr(b, "out"))
        shim(b)(p(arr(b, "A")), p(arr(b, "B")), p(o), o.shape[0])
        assert_f16_gemm_close(o, arr(b, "out"))
    for b in ("fp16_matmul_hmx_deepk", "fp16_matmul_leaky_relu_hmx"):
        o = np.zeros_like(arr(b, "out"))
        shim(b)(p(arr(b, "A")), p(arr(b, "B")), p(o), o.shape[0], arr(b, "A").shape[1])
        assert_f16_gemm_close(o, arr(b, "out"))
    b = "hmx_matmul_fp16_bias"
    o = np.zeros_like(arr(b, "out"))
    shim(b)(p(arr(b, "A")), p(arr(b, "B")), p(arr(b, "bias")), p(o), o.shape[0])
    assert_f16_gemm_close(o, arr(b, "out"))
    b = "hmx_tile_mac_fp16_32"
    o = arr(b, "C").copy()
    shim(b)(p(arr(b, "A")), p(arr(b, "B")), p(o), o.shape[0])
    assert_f16_gemm_close(o, arr(b, "out"))
    b = "av_tile_fp16"
    (M, N), D = arr(b, "A").shape, arr(b, "V").shape[0]
    o = np.zeros_like(arr(b, "out"))
    shim(b)(p(arr(b, "A")), p(arr(b, "V")), p(o), M, N, D)
    assert_f16_gemm_close(o, arr(b, "out"))


def test_shim_i8_callers(hx):
    from conftest import golden
    g = golden("i8_callers")
    c = lambda a: np.ascontiguousarray(a)
    M, N = g["gbr_out"].shape
    K = g["gbr_A"].shape[1]
    o = np.zeros((M, N), np.int8)
    shim("gemm_bias_relu_requant")(p(c(g["gbr_A"])), p(c(g["gbr_B"])), p(c(g["gbr_bias"])), p(o), M, N, K,
                                   C.c_int32(1 << 30), 38, C.c_int8(3))
    np.testing.assert_array_equal(o, g["gbr_out"])
    M, K = g["mv_A"].shape
    for name in ("i8_linear_relu_requant", "i8_matvec_bias_requant"):
        o = np.zeros(M, np.int8)
        shim(name)(p(c(g["mv_A"])), p(c(g["mv_x"])), p(c(g["mv_bias"])), p(o), M, K, C.c_int32(1 << 30), 38,
                   C.c_int8(-2))
        np.testing.assert_array_equal(o, g[name + "_out"])
    n = g["c11_out"].shape[0]
    o = np.zeros((n, n), np.int32)
    shim("hmx_conv1x1_i8")(p(c(g["c11_In"])), p(c(g["c11_W"])), p(c(g["c11_bias"])), p(o), n)
    np.testing.assert_array_equal(o, g["c11_out"])
    M, N = g["tbr_out"].shape
    K = g["tbr_A"].shape[1]
    o = np.zeros((M, N), np.uint8)
    shim("i8_gemm_tiled_bias_relu_requant")(p(c(g["tbr_A"])), p(c(g["tbr_B"])), p(c(g["tbr_bias"])), p(o),
                                            M, N, K)
    np.testing.assert_array_equal(o, g["tbr_out"])
    for name in ("i8_conv2d_1x1_hmx", "i8_pointwise_conv_hmx"):
        o = np.zeros((64, 64), np.uint16)
        shim(name)(p(c(g[name + "_in"])), p(c(g[name + "_W"])), p(o), 64)
        np.testing.assert_array_equal(o, g[name + "_out"])
