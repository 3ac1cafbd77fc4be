"""Integer row operators on the B200 (table layernorms, exp-table softmaxes,
int16 and double requants, GEMM + softmax tiles, the GELU FFN block),
bit-exact against the reference's outputs (golden int_rows) and the oracle
on larger and ragged shapes; the shims of the bundles whose harnesses need
the Hexagon SDK on their golden cases."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from test_oracle_golden import NORM_MULT, NORM_SHIFT, int_rows_calls

pytestmark = pytest.mark.gpu

SHIMS = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"


def test_int_rows_golden(hx):
    for k, (got, exp) in enumerate(int_rows_calls(hx, golden("int_rows"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def test_sdk_harness_bundles_through_shims(hx, oracle):
    g = golden("int_rows")
    n = "i8_layernorm_dma"
    x = g[n + "__x"]
    out = np.zeros_like(x)
    shim(n)(p(x), p(out), x.shape[0], x.shape[1], p(g[n + "__gamma"]), p(g[n + "__beta"]), p(g["inv_lut"]))
    np.testing.assert_array_equal(out, g[n + "__out"])
    n = "i8_norm_requant_dma"
    x = g[n + "__x"]
    out = np.zeros_like(x)
    shim(n)(p(x), p(out), x.size)
    np.testing.assert_array_equal(out, g[n + "__out"])
    rng = np.random.default_rng(9)
    x16 = rng.integers(-20000, 20000, (33, 517)).astype(np.int16)
    lut16 = rng.integers(0, 65536, 256).astype(np.uint16)
    out16 = np.zeros_like(x16)
    shim("vtcm_softmax_row_i16")(p(x16), p(out16), 33, 517, p(lut16))
    np.testing.assert_array_equal(out16, oracle.lut_softmax_i16(x16, lut16))


@pytest.mark.parametrize("R,W", [(1, 1), (7, 33), (300, 200), (4096, 64), (65, 4099)])
def test_layernorm_lut_i8_random(hx, oracle, R, W):
    rng = np.random.default_rng(R * 3 + W)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    x, res = s8(R, W), s8(R, W)
    inv = rng.integers(0, 256, 256, dtype=np.uint8)
    g, b = s8(W), s8(W)
    for kw in (dict(), dict(res=res)):
        np.testing.assert_array_equal(hx.layernorm_lut_i8(x, g, b, inv, **kw),
                                      oracle.layernorm_lut_i8(x, g, b, inv, **kw))
    gr, br = s8(R * W), s8(R * W)
    np.testing.assert_array_equal(hx.layernorm_lut_i8(x, gr, br, inv, "rowwise"),
                                  oracle.layernorm_lut_i8(x, gr, br, inv, "rowwise"))
    gp, bp, lp = s8(R), s8(R), rng.integers(0, 256, (R, 256), dtype=np.uint8)
    np.testing.assert_array_equal(hx.layernorm_lut_i8(x, gp, bp, lp, "per_row"),
                                  oracle.layernorm_lut_i8(x, gp, bp, lp, "per_row"))
    idx = rng.integers(0, R, 3 * R + 1).astype(np.int32)
    np.testing.assert_array_equal(hx.layernorm_lut_i8(x, g, b, inv, idx=idx),
                                  oracle.layernorm_lut_i8(x, g, b, inv, idx=idx))


@pytest.mark.parametrize("R,C", [(1, 1), (9, 300), (2048, 256), (3, 10000)])
def test_layernorm_lut_i16_and_softmaxes(hx, oracle, R, C):
    rng = np.random.default_rng(R + C)
    x = rng.integers(-32768, 32768, (R, C)).astype(np.int16)
    inv = rng.integers(0, 65536, 256).astype(np.uint16)
    gc, bc = (rng.integers(-1024, 1025, C).astype(np.int16), rng.integers(-32768, 32768, C).astype(np.int16))
    gr, br = (rng.integers(-1024, 1025, R).astype(np.int16), rng.integers(-32768, 32768, R).astype(np.int16))
    np.testing.assert_array_equal(hx.layernorm_lut_i16(x, gc, bc, inv, 0), oracle.layernorm_lut_i16(x, gc, bc, inv, 0))
    np.testing.assert_array_equal(hx.layernorm_lut_i16(x, gr, br, inv, 1), oracle.layernorm_lut_i16(x, gr, br, inv, 1))
    lut16 = rng.integers(0, 65536, 256).astype(np.uint16)
    lut16[255] |= 1
    np.testing.assert_array_equal(hx.lut_softmax_i16(x, lut16), oracle.lut_softmax_i16(x, lut16))
    x8 = rng.integers(-128, 128, (R, C), dtype=np.int8)
    lut8 = rng.integers(0, 256, 256, dtype=np.uint8)
    lut8[255] |= 1
    np.testing.assert_array_equal(hx.lut_softmax_u8(x8, lut8), oracle.lut_softmax_u8(x8, lut8))


def test_requants_and_compositions(hx, oracle):
    rng = np.random.default_rng(17)
    a = rng.integers(-2**31, 2**31, (1 << 22) + 7, dtype=np.int64).astype(np.int32)
    for mult, shift in ((1 << 20, 30), (-77777, 9), (1, 0), (2**31 - 1, 63)):
        np.testing.assert_array_equal(hx.requant_i16(a, mult, shift), oracle.requant_i16(a, mult, shift))
    x = rng.integers(-128, 128, 16 * 100003 + 11, dtype=np.int8)
    np.testing.assert_array_equal(hx.norm_requant_i8(x, NORM_MULT, NORM_SHIFT, 5, 4, 0),
                                  oracle.norm_requant_i8(x, NORM_MULT, NORM_SHIFT, 5, 4, 0))
    A, B = (rng.integers(-128, 128, (300, 256), dtype=np.int8), rng.integers(-128, 128, (256, 520), dtype=np.int8))
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    lut[255] |= 1
    np.testing.assert_array_equal(hx.gemm_softmax_u8(A, B, lut), oracle.gemm_softmax_u8(A, B, lut))
    Bt = np.ascontiguousarray(B.T)
    np.testing.assert_array_equal(hx.gemm_softmax_u8(A, Bt, lut, True, True, 3000, 14),
                                  oracle.gemm_softmax_u8(A, Bt, lut, True, True, 3000, 14))
    M, K, V, D = 200, 128, 256, 96
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    args = (s8(M, K), s8(K, V), rng.integers(-3000, 3000, V).astype(np.int32), s8(256), s8(V, D),
            rng.integers(-3000, 3000, D).astype(np.int32), s8(M, D), s8(D), s8(D),
            rng.integers(0, 256, 256, dtype=np.uint8))
    np.testing.assert_array_equal(hx.gelu_ffn_residual_i8(*args), oracle.gelu_ffn_residual_i8(*args))


from test_oracle_golden import check_softmax_rms  # noqa: E402


def test_softmax_rms_golden(hx):
    check_softmax_rms(hx, golden("softmax_rms"))


def test_softmax_recip_and_rms_random(hx, oracle):
    rng = np.random.default_rng(21)
    x = rng.integers(-128, 128, (1000, 777), dtype=np.int8)
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    rl = rng.integers(0, 65536, 256, dtype=np.uint16)
    np.testing.assert_array_equal(hx.lut_softmax_u8(x, lut, rl), oracle.lut_softmax_u8(x, lut, rl))
    g = rng.integers(-128, 128, 777, dtype=np.int8)
    inv = rng.integers(0, 256, 256, dtype=np.uint8)
    np.testing.assert_array_equal(hx.layernorm_lut_i8(x, g, None, inv, "rms", res=x[::-1].copy()),
                                  oracle.layernorm_lut_i8(x, g, None, inv, "rms", res=x[::-1].copy()))
    xf = rng.standard_normal((300, 4096)).astype(np.float16)
    gain = rng.standard_normal(300).astype(np.float16)
    got = hx.rmsnorm_gain_f16(xf, gain, 1e-3).astype(np.float64)
    exp = oracle.rmsnorm_gain_f16(xf, gain, 1e-3).astype(np.float64)
    assert np.all(np.abs(got - exp) <= 1e-2 * np.abs(exp) + 1e-3 * np.abs(exp).max())


def test_attention_qkt_tile_shim(hx):
    """attention_qkt_tile's own harness reads past its parameter tables, so
    its shim is checked here on the golden case (valid scale parameters)."""
    g = golden("int_rows")
    Q, K, exp = (g["attention_qkt_tile__" + k] for k in ("Q", "K", "out"))
    out = np.zeros_like(exp)
    fn = shim("attention_qkt_tile")
    fn.argtypes = [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_int32, C.c_int]
    fn(p(Q), p(K), p(out), Q.shape[0], K.shape[0], Q.shape[1], 1 << 20, 26)
    np.testing.assert_array_equal(out, exp)


from test_oracle_golden import sparse_attn_calls  # noqa: E402


def test_sparse_attn_golden_and_shim(hx):
    g = golden("sparse_attn")
    for got, exp in sparse_attn_calls(hx, g):
        np.testing.assert_array_equal(got, exp)
    fn = shim("i8_sparse_attn_block")
    fn.argtypes = [C.c_void_p] * 5 + [C.c_int, C.c_int32, C.c_int, C.c_int32, C.c_int]
    for t in range(8):
        w, sm, ss, am, ash = (int(v) for v in g[f"params{t}"])
        out = np.zeros((1, 8, 16), np.int8)
        fn(p(g[f"Q{t}"]), p(g[f"K{t}"]), p(g[f"V{t}"]), p(g[f"lut{t}"]), p(out), w, sm, ss, am, ash)
        np.testing.assert_array_equal(out, g[f"out{t}"])


@pytest.mark.parametrize("H,S,D", [(1, 1, 1), (4, 33, 20), (16, 128, 64)])
def test_sparse_attn_random(hx, oracle, H, S, D):
    rng = np.random.default_rng(H * S + D)
    Q, K, V = (rng.integers(-128, 128, (H, S, D), dtype=np.int8) for _ in range(3))
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    lut[255] = 255
    for w in (0, 1, 5, S):
        for sm, ss, am, ash in ((3, 7, 5, 8), (1 << 12, 17, 77, 14)):
            np.testing.assert_array_equal(hx.attn_lut_i8_window(Q, K, V, lut, w, sm, ss, am, ash),
                                          oracle.attn_lut_i8_window(Q, K, V, lut, w, sm, ss, am, ash))


from test_oracle_golden import cache_rope_calls  # noqa: E402


def test_cache_rope_golden_and_shims(hx):
    g = golden("cache_rope")
    for got, exp in cache_rope_calls(hx, g):
        np.testing.assert_array_equal(got.view(np.uint8), exp.view(np.uint8))
    fn = shim("kv_cache_update")
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int] * 4
    for t in range(3):
        kc, vc = g[f"kc{t}"].copy(), g[f"vc{t}"].copy()
        heads, cl, hd = kc.shape
        fn(p(kc), p(vc), p(g[f"kn{t}"]), p(g[f"vn{t}"]), int(g[f"pos{t}"]), heads, cl, hd)
        np.testing.assert_array_equal(kc, g[f"kout{t}"])
        np.testing.assert_array_equal(vc, g[f"vout{t}"])
    fn = shim("rope_pair_fp16")
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int]
    for t in range(2):
        x = g[f"x{t}"]
        out = np.zeros_like(x)
        fn(p(x), p(g[f"cos{t}"]), p(g[f"sin{t}"]), p(out), x.size // 2)
        np.testing.assert_array_equal(out.view(np.uint16), g[f"rope{t}"].view(np.uint16))


@pytest.mark.parametrize("heads,cl,hd,pos", [(1, 1, 1, 0), (32, 4096, 128, 4095), (7, 300, 20, 123)])
def test_kv_cache_update_random(hx, oracle, heads, cl, hd, pos):
    rng = np.random.default_rng(heads + hd)
    kc, vc = (rng.integers(-128, 128, (heads, cl, hd), dtype=np.int8) for _ in range(2))
    kn, vn = (rng.integers(-128, 128, (heads, hd), dtype=np.int8) for _ in range(2))
    ek, ev = oracle.kv_cache_update_i8(kc, vc, kn, vn, pos)
    gk, gv = hx.kv_cache_update_i8(kc.copy(), vc.copy(), kn, vn, pos)
    np.testing.assert_array_equal(gk, ek)
    np.testing.assert_array_equal(gv, ev)
    with pytest.raises(RuntimeError):
        hx.kv_cache_update_i8(kc, vc, kn, vn, cl)


def test_rope_pair_random(hx, oracle):
    rng = np.random.default_rng(41)
    n = (1 << 22) + 3
    x = (rng.standard_normal(2 * n) * 30).astype(np.float16)
    th = rng.uniform(-np.pi, np.pi, n)
    c, s = np.cos(th).astype(np.float16), np.sin(th).astype(np.float16)
    np.testing.assert_array_equal(hx.rope_pair_f16(x, c, s).view(np.uint16),
                                  oracle.rope_pair_f16(x, c, s).view(np.uint16))


from test_oracle_golden import block_calls  # noqa: E402


def test_blocks_golden_and_shims(hx):
    g = golden("blocks")
    for k, (got, exp) in enumerate(block_calls(hx, g)):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))
    for t in range(2):
        c = lambda k: g[f"ffn_{k}{t}"]
        S, D = c("X").shape
        out = np.zeros((S, D), np.int8)
        shim("i8_ffn_block")(p(c("X")), p(c("W1")), p(c("b1")), p(c("W2")), p(c("b2")), p(out), S, D,
                             c("W1").shape[1])
        np.testing.assert_array_equal(out, c("out"))
        c = lambda k: g[f"sw_{k}{t}"]
        S, D = c("X").shape
        out = np.zeros((S, D), np.int8)
        shim("i8_ffn_swiglu_block")(p(c("X")), p(c("Wg")), p(c("Wu")), p(c("Wd")), p(c("bd")), p(c("lut")),
                                    p(out), S, D, c("Wg").shape[1])
        np.testing.assert_array_equal(out, c("out"))
        c = lambda k: g[f"enc_{k}{t}"]
        S, D = c("X").shape
        out = np.zeros((S, D), np.int8)
        shim("i8_transformer_encoder_block")(p(c("X")), p(c("W1")), p(c("b1")), p(c("W2")), p(c("b2")),
                                             p(c("lut")), p(out), S, D, c("W1").shape[1])
        np.testing.assert_array_equal(out, c("out"))


@pytest.mark.parametrize("M,D,F", [(1, 1, 1), (1000, 256, 512), (333, 130, 70)])
def test_hmx_ffns_random(hx, oracle, M, D, F):
    rng = np.random.default_rng(M + D + F)
    X = rng.integers(0, 256, (M, D), dtype=np.uint8)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    W1, W2, Wu = s8(D, F), s8(F, D), s8(D, F)
    b1 = rng.integers(-3000, 3000, F).astype(np.int32)
    b2 = rng.integers(-3000, 3000, D).astype(np.int32)
    np.testing.assert_array_equal(hx.ffn_hmx_i8(X, W1, b1, W2, b2), oracle.ffn_hmx_i8(X, W1, b1, W2, b2))
    np.testing.assert_array_equal(hx.ffn_hmx_i8(X, W1, b1, W2, b2, 5, 7),
                                  oracle.ffn_hmx_i8(X, W1, b1, W2, b2, 5, 7))
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    args = (X, W1, Wu, W2, b2, lut)
    np.testing.assert_array_equal(hx.ffn_swiglu_hmx_i8(*args), oracle.ffn_swiglu_hmx_i8(*args))
    np.testing.assert_array_equal(hx.ffn_swiglu_hmx_i8(*args, 3, 1, 6, 100, 2),
                                  oracle.ffn_swiglu_hmx_i8(*args, 3, 1, 6, 100, 2))


@pytest.mark.parametrize("S,D,F", [(1, 1, 1), (64, 64, 128), (31, 45, 77), (96, 128, 192)])
def test_encoder_block_random(hx, oracle, S, D, F):
    rng = np.random.default_rng(S * D + F)
    X = rng.integers(0, 256, (S, D), dtype=np.uint8)
    W1 = rng.integers(-128, 128, (D, F), dtype=np.int8)
    W2 = rng.integers(-128, 128, (F, D), dtype=np.int8)
    b1 = rng.integers(-3000, 3000, F).astype(np.int32)
    b2 = rng.integers(-3000, 3000, D).astype(np.int32)
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    lut[255] = 255
    np.testing.assert_array_equal(hx.encoder_block_i8(X, W1, b1, W2, b2, lut),
                                  oracle.encoder_block_i8(X, W1, b1, W2, b2, lut))
