"""tcgen05 GEMMs and requant kernels on the B200 vs the reference.

Integer paths are bit-exact against the reference's golden outputs and the
oracle.  fp16 GEMMs: |got - exp| <= 1e-2 * |exp| + 1e-3 * max|exp| against the
fp32-accumulating reference (in practice at most 1 fp16 ulp apart).
"""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------- requant kernels

def test_requant_per_channel_golden(hx):
    g = golden("requant_per_channel_harness")
    R, Cc = g["dims"]
    a = g["a"].reshape(R, Cc)
    for k in range(len(g["zp"])):
        out = hx.requant_per_channel(a, g["mult"][k], g["shift"][k], int(g["zp"][k]))
        np.testing.assert_array_equal(out.ravel(), g["out"][k])


def test_requantize_i32_u8_golden(hx):
    g = golden("requantize_i32_u8_harness")
    n = 262144
    i = np.arange(n, dtype=np.int64)
    a = (((i * 2731 + 5) & 0xFFFF) - 32768).astype(np.int32)
    a[:6] = [32767, -32768, 0, 6400, 13000, -13000]
    for p, (mult, shift, zp) in enumerate(g["params"]):
        np.testing.assert_array_equal(hx.requantize_i32_u8(a, int(mult), int(shift), int(zp)),
                                      g["out"][p])
    # ragged length and misaligned start take the scalar path
    out = hx.requantize_i32_u8(a[3:100003], 5, 8, 128)
    np.testing.assert_array_equal(out, g["out"][0][3:100003])


# ------------------------------------------------------------- int8 GEMMs

def test_i8_gemm_requant_harness(hx):
    g = golden("i8_gemm_requant_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = hx.gemm_i8_requant(A, B, int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_i8_gemm_requant_256_config(hx):
    """int8 x int8 -> int32 GEMM M=N=K=256 (seed 0) and its rounding sweep."""
    g = golden("i8_gemm_requant_256")
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = hx.gemm_i8_requant(g["A"], g["B"], int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out, g["out"][p])


def test_i8_gemm_bias_requant_harness(hx):
    g = golden("i8_gemm_bias_requant_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = hx.gemm_i8_bias_requant(A, B, g["bias"], int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_gemm_tile_zp_i8_harness(hx):
    g = golden("gemm_tile_zp_i8_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (zpa, mult, shift) in enumerate(g["params"]):
        out = hx.gemm_i8_zp(A, B, int(zpa), int(mult), int(shift))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_gemm_u8s8_pc_golden(hx):
    g = golden("gemm_u8s8_pc_small")
    for c in range(int(g["ncases"])):
        k = lambda s: g[f"c{c}_{s}"]
        out = hx.gemm_u8s8_pc(k("A"), k("B"), k("bias"), int(k("zpa")), k("mult"), k("shift"),
                              int(k("zp_out")))
        np.testing.assert_array_equal(out, k("out"))


I8_SHAPES = [(1, 1, 1), (1, 300, 17), (129, 257, 130), (256, 384, 512), (200, 64, 0),
             (300, 520, 1000), (128, 256, 4096), (513, 129, 96)]


@pytest.mark.parametrize("M,N,K", I8_SHAPES)
def test_gemm_u8s8_pc_random(hx, oracle, M, N, K):
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = rng.integers(30, 46, N).astype(np.int32)
    for zpa in (128, 0, -7):
        got = hx.gemm_u8s8_pc(A, B, bias, zpa, mult, shift, 128)
        exp = oracle.gemm_u8s8_pc(A, B, bias, zpa, mult, shift, 128)
        np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("M,N,K", I8_SHAPES)
def test_gemm_i8_variants_random(hx, oracle, M, N, K):
    rng = np.random.default_rng(M + N * 3 + K * 5)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = rng.integers(-40000, 40000, N).astype(np.int32)
    for mult, shift, zp in ((1, 0, 0), (3, 5, -2), (1234567, 30, 4), (2**31 - 1, 40, 0)):
        np.testing.assert_array_equal(hx.gemm_i8_requant(A, B, mult, shift, zp),
                                      oracle.gemm_i8_requant(A, B, mult, shift, zp))
        np.testing.assert_array_equal(hx.gemm_i8_bias_requant(A, B, bias, mult, shift, zp),
                                      oracle.gemm_i8_bias_requant(A, B, bias, mult, shift, zp))
        np.testing.assert_array_equal(hx.gemm_i8_zp(A, B, -13, mult, shift),
                                      oracle.gemm_i8_zp(A, B, -13, mult, shift))


def test_gemm_u8s8_extreme_values(hx, oracle):
    # all-max / all-min operands: largest |acc| the shape allows
    M, N, K = 130, 200, 2048
    A = np.full((M, K), 255, np.uint8)
    A[::2] = 0
    B = np.full((K, N), -128, np.int8)
    B[:, ::3] = 127
    bias = np.zeros(N, np.int32)
    mult = np.full(N, 2**31 - 1, np.int32)
    shift = np.full(N, 40, np.int32)
    np.testing.assert_array_equal(hx.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128),
                                  oracle.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128))


# ------------------------------------------------- HMX-convention GEMMs

from test_oracle_golden import HMX_CASES, hmx_case  # noqa: E402


@pytest.mark.parametrize("tag,kind,bt", HMX_CASES)
def test_hmx_gemm_golden(hx, tag, kind, bt):
    A, B, out, K, N, zp, bias = hmx_case(golden("hmx_gemm"), tag)
    B = B.reshape((N, K) if bt else (K, N))
    np.testing.assert_array_equal(hx.gemm_hmx(A, B, kind, bias, zp, bt), out)


@pytest.mark.parametrize("M,N,K", I8_SHAPES)
def test_hmx_gemm_random(hx, oracle, M, N, K):
    rng = np.random.default_rng(M * 5 + N * 11 + K)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    Bt = np.ascontiguousarray(B.T)
    bias = rng.integers(-3000, 3000, N).astype(np.int32)
    for kind in (0, 1, 2):
        for zpa in (0, 128, -5):
            exp = oracle.gemm_hmx(A, B, kind, bias, zpa)
            np.testing.assert_array_equal(hx.gemm_hmx(A, B, kind, bias, zpa), exp)
            np.testing.assert_array_equal(hx.gemm_hmx(A, Bt, kind, bias, zpa, True), exp)


def test_hmx_gemm_deep_k_wraps(hx, oracle):
    """K = 8192 full-range operands: acc * 17 leaves int32, so the 12-bit
    field wraps; the int32 two's-complement arithmetic must agree."""
    M, N, K = 256, 384, 8192
    rng = np.random.default_rng(7)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    for zpa in (0, 128):
        exp = oracle.gemm_hmx(A, B, 0, None, zpa)
        np.testing.assert_array_equal(hx.gemm_hmx(A, B, 0, None, zpa), exp)
        np.testing.assert_array_equal(
            hx.gemm_hmx(A, np.ascontiguousarray(B.T), 0, None, zpa, True), exp)


from hmx_family import BUNDLES as HMX_FAMILY, golden_case  # noqa: E402


@pytest.mark.parametrize("bundle", sorted(HMX_FAMILY))
def test_hmx_family_golden(hx, bundle):
    A, B, out, kw = golden_case(golden("hmx_family"), bundle)
    np.testing.assert_array_equal(hx.gemm_hmx_ex(A, B, **kw), out)


HMX_EX_SHAPES = [(1, 1, 1), (129, 257, 130), (300, 520, 1000), (513, 129, 96), (256, 384, 4096)]


@pytest.mark.parametrize("M,N,K", HMX_EX_SHAPES)
def test_hmx_ex_random(hx, oracle, M, N, K):
    """Every store kind and activation, with bias, int32 / int8 residuals,
    column-major output, Bt operand and a zero point, against the oracle."""
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    Bt = np.ascontiguousarray(B.T)
    bias = rng.integers(-3000, 3000, N).astype(np.int32)
    r32 = rng.integers(-10**6, 10**6, (M, N)).astype(np.int32)
    r8 = rng.integers(-128, 128, (M, N)).astype(np.int8)
    l32 = rng.integers(-10**5, 10**5, 256).astype(np.int32)
    l8 = rng.integers(-128, 128, 256).astype(np.int8)
    cases = [dict(store="i32", act="leaky_shr3", bias=bias, res=r32),
             dict(store="i8_sat", res=r8, zpA=128),
             dict(store="u8_sat", act="relu", bias=bias),
             dict(store="i8_low", zpA=-3),
             dict(store="u16_field", col_major=True),
             dict(store="lut_i32", lut=l32, bias=bias),
             dict(store="lut_i8", lut=l8, bias=bias, res=r8),
             dict(store="i32", act="relu", col_major=True, res=r32, zpA=7)]
    for kw in cases:
        exp = oracle.gemm_hmx_ex(A, B, **kw)
        np.testing.assert_array_equal(hx.gemm_hmx_ex(A, B, **kw), exp, err_msg=str(kw.keys()))
        np.testing.assert_array_equal(hx.gemm_hmx_ex(A, Bt, b_transposed=True, **kw), exp)


def test_int8_attention_hmx_golden(hx):
    g = golden("int8_attention_hmx")
    S, D = g["qkt_SD"]
    np.testing.assert_array_equal(
        hx.gemm_hmx_ex(g["qkt_Q"].reshape(S, D), g["qkt_K"].reshape(S, D), "u16_field",
                       b_transposed=True), g["qkt_out"].reshape(S, S))
    np.testing.assert_array_equal(
        hx.gemm_hmx_ex(g["av_P"].reshape(S, S), g["av_V"].reshape(S, D), "u16_field"),
        g["av_out"].reshape(S, D))
    S, D = g["qkav_SD"]
    np.testing.assert_array_equal(
        hx.attn_qkt_av_hmx(g["qkav_Q"].reshape(S, D), g["qkav_K"].reshape(S, D),
                           g["qkav_V"].reshape(S, D)), g["qkav_out"].reshape(S, D))


@pytest.mark.parametrize("SQ,SK,D", [(1, 1, 1), (32, 32, 32), (300, 200, 96), (129, 1000, 64),
                                     (517, 384, 128)])
def test_attn_qkt_av_hmx_random(hx, oracle, SQ, SK, D):
    """The byte-split second product against the oracle's direct int sum,
    full-range inputs (Sc spans the whole 12-bit field)."""
    rng = np.random.default_rng(SQ + SK + D)
    Q = rng.integers(0, 256, (SQ, D), dtype=np.uint8)
    K = rng.integers(-128, 128, (SK, D), dtype=np.int8)
    V = rng.integers(-128, 128, (SK, D), dtype=np.int8)
    np.testing.assert_array_equal(hx.attn_qkt_av_hmx(Q, K, V), oracle.attn_qkt_av_hmx(Q, K, V))


# --------------------------------------------------------------- fp16 GEMMs

def assert_f16_gemm_close(got, exp):
    g, e = got.astype(np.float64), exp.astype(np.float64)
    lim = 1e-2 * np.abs(e) + 1e-3 * np.abs(e).max()
    bad = np.abs(g - e) > lim
    assert not bad.any(), f"{bad.sum()} of {bad.size} off"
    # both sides are one fp16 rounding of an fp32 sum; the sums differ only by
    # accumulation order, so almost every element is within 1 fp16 ulp (the
    # rest are near-zero outputs of deep-K cancellation)
    ulp = np.abs(got.view(np.int16).astype(np.int32) - exp.view(np.int16).astype(np.int32))
    assert np.mean(ulp <= 1) > 0.99


@pytest.mark.parametrize("name,kind", [("gemm_f16_nt_harness", "nt"),
                                       ("gemm_f16_nn_harness", "nn"),
                                       ("attn_av_f16_harness", "nn")])
def test_f16_gemm_harness_golden(hx, name, kind):
    g = golden(name)
    M, N, K = g["dims"]
    if kind == "nt":
        got = hx.gemm_f16_nt(g["A"].reshape(M, K), g["Bt"].reshape(N, K))
    else:
        got = hx.gemm_f16_nn(g["A"].reshape(M, K), g["B"].reshape(K, N))
    # the harnesses' own deep-K tolerance (atol 8e-3, rtol 1.2e-2)
    e = g["out"].astype(np.float32).reshape(M, N)
    assert np.all(np.abs(got.astype(np.float32) - e) <= 8e-3 + 1.2e-2 * np.abs(e))
    assert_f16_gemm_close(got, g["out"].reshape(M, N))


@pytest.mark.parametrize("name", ["gemm_f16_nt_256x512", "gemm_f16_nt_192x320"])
def test_f16_gemm_multi_tile_golden(hx, name):
    g = golden(name)
    assert_f16_gemm_close(hx.gemm_f16_nt(g["A"], g["Bt"]), g["out"])


F16_SHAPES = [(1, 1, 1), (7, 300, 24), (129, 257, 130), (256, 512, 1024), (384, 128, 64),
              (300, 520, 1000), (128, 256, 8192), (1000, 40, 77)]


@pytest.mark.parametrize("M,N,K", F16_SHAPES)
def test_f16_gemm_random(hx, oracle, M, N, K):
    rng = np.random.default_rng(M * 13 + N + K * 3)
    A = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    Bt = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)
    assert_f16_gemm_close(hx.gemm_f16_nt(A, Bt), oracle.gemm_f16_nt(A, Bt))
    B = np.ascontiguousarray(Bt.T)
    assert_f16_gemm_close(hx.gemm_f16_nn(A, B), oracle.gemm_f16_nn(A, B))


# ------------------------------------------------- benchmark configurations

def fp32_matmul_ieee():
    """torch fp32 matmuls of the checkers in full fp32 (no TF32)."""
    import torch
    try:
        torch.backends.cuda.matmul.fp32_precision = "ieee"
    except AttributeError:
        torch.backends.cuda.matmul.allow_tf32 = False


def _crc_inputs(kind):
    import sys

    from conftest import GOLDEN
    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    import make_crc
    return make_crc, make_crc.inputs(kind)


@pytest.mark.slow
def test_u8s8_benchmark_shape(hx):
    """u8 x s8 GEMM M=16384, N=K=8192 (zpA 128, bias N(0,1000), per-channel
    mult/shift 44, zp_out 128): the WHOLE GPU output bit-exact against the
    oracle, through per-row CRC32s of the oracle's output made offline by
    tests/golden/make_crc.py; output spread over the u8 range."""
    mk, d = _crc_inputs("u8s8")
    got = hx.gemm_u8s8_pc(d["A"], d["B"], d["bias"], d["zpA"], d["mult"], d["shift"], d["zp_out"])
    exp = np.load(mk.FILES["u8s8"])
    crc = mk.row_crcs(got)
    bad = np.flatnonzero(crc != exp)
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:8]}"
    assert 20 < got.std() < 100


@pytest.mark.slow
def test_hmx_benchmark_shape(hx):
    """HMX-convention u8 x s8 GEMM M=16384, N=K=8192, sx12 field + bias,
    ReLU, int32 out: the WHOLE output bit-exact against the oracle's per-row
    CRC32s."""
    mk, d = _crc_inputs("hmx")
    got = hx.gemm_hmx_ex(d["A"], d["B"], "i32", "relu", bias=d["bias"])
    exp = np.load(mk.FILES["hmx"])
    bad = np.flatnonzero(mk.row_crcs(got) != exp)
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:8]}"
    assert (got > 0).mean() > 0.3


def _dev_gemm(kind, d, rows):
    """One device-pointer launch over rows [0, rows) of the benchmark inputs
    (the per-rank problem of an 8-way row split when rows = 2048)."""
    import torch

    from hexkernels_b200 import _lib
    lib = _lib.load()
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items()
         if isinstance(v, np.ndarray)}
    A = t["A"][:rows].contiguous()
    K, N = d["B"].shape
    if kind == "u8s8":
        out = torch.empty((rows, N), dtype=torch.uint8, device="cuda")
        _lib.check(lib.hexcuda_gemm_u8s8_pc(0, A.data_ptr(), t["B"].data_ptr(),
                                            t["bias"].data_ptr(), out.data_ptr(), rows, N, K,
                                            d["zpA"], t["mult"].data_ptr(), t["shift"].data_ptr(),
                                            d["zp_out"]))
    else:
        out = torch.empty((rows, N), dtype=torch.int32, device="cuda")
        _lib.check(lib.hexcuda_gemm_hmx_ex(0, A.data_ptr(), t["B"].data_ptr(), 0,
                                           t["bias"].data_ptr(), None, 0, None, out.data_ptr(),
                                           hx_store("i32"), hx_act("relu"), 0, rows, N, K, 0))
    _lib.check(lib.hexcuda_sync(0))
    return out.cpu().numpy()


def hx_store(name):
    from hexkernels_b200 import ops
    return ops.HMX_STORE[name][0]


def hx_act(name):
    from hexkernels_b200 import ops
    return ops.HMX_ACT[name]


@pytest.mark.slow
@pytest.mark.parametrize("kind", ["u8s8", "hmx"])
def test_split_tail_at_eight_way_shard(hx, kind):
    """2048 x 8192 x 8192 (the benchmark GEMMs' per-rank rows at 8 GPUs):
    512 one-SM tiles for u8s8, whose last wave is cut into two K parts per
    tile; 256 CTA-pair tiles for HMX (not split behind full waves).  Rows
    0..2047 must equal the oracle's per-row CRC32s of the full benchmark
    output."""
    mk, d = _crc_inputs(kind)
    got = _dev_gemm(kind, d, 2048)
    exp = np.load(mk.FILES[kind])[:2048]
    bad = np.flatnonzero(mk.row_crcs(got) != exp)
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:8]}"


def test_split_tail_small_shapes_exact(hx, oracle):
    """Fewer tiles than SMs with a deep K: every tile is cut into K parts
    (u8s8 128 x 256 tiles: 4 tiles, 4 parts over 33 K blocks, ragged; HMX
    CTA pairs: 4 pair tiles, 2 parts) and merged exactly."""
    rng = np.random.default_rng(21)
    M, N, K = 256, 384, 4224
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 3000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = rng.integers(38, 44, N).astype(np.int32)
    np.testing.assert_array_equal(hx.gemm_u8s8_pc(A, B, bias, 77, mult, shift, 128),
                                  oracle.gemm_u8s8_pc(A, B, bias, 77, mult, shift, 128))
    M, N, K = 512, 512, 2048
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = rng.integers(-3000, 3000, N).astype(np.int32)
    res = rng.integers(-128, 128, (M, N), dtype=np.int8)
    for kw in (dict(store="i32", act="relu", bias=bias), dict(store="i8_sat", res=res, zpA=9),
               dict(store="acc_i32")):
        np.testing.assert_array_equal(hx.gemm_hmx_ex(A, B, **kw), oracle.gemm_hmx_ex(A, B, **kw),
                                      err_msg=str(sorted(kw)))
    # s8 x s8 requant GEMM: 2 row tiles of one 256-column tile, 2 parts
    A8 = rng.integers(-128, 128, (256, 2048), dtype=np.int8)
    B8 = rng.integers(-128, 128, (2048, 256), dtype=np.int8)
    got = hx.gemm_i8_requant(A8, B8, 1 << 30, 42, 3)
    np.testing.assert_array_equal(got, oracle.gemm_i8_requant(A8, B8, 1 << 30, 42, 3))
    assert 20 < got.std() < 100


def test_f16_gemm_never_split(hx):
    """fp16 GEMMs with fewer tiles than SMs and a deep K are not cut into K
    parts: a 100-row launch gives the same bits as the same rows inside a
    16-row-tile launch (one-SM kernel) and a 512-row launch (CTA pairs)."""
    rng = np.random.default_rng(22)
    K, N = 8192, 512
    A = (rng.standard_normal((2048, K)) / np.sqrt(K)).astype(np.float16)
    Bt = rng.standard_normal((N, K)).astype(np.float16)
    full = hx.gemm_f16_nt(A, Bt)
    np.testing.assert_array_equal(hx.gemm_f16_nt(A[:100], Bt), full[:100])
    np.testing.assert_array_equal(hx.gemm_f16_nt(A[:512], Bt), full[:512])


@pytest.mark.slow
def test_f16_benchmark_shape(hx, oracle):
    """fp16 GEMM M=N=K=8192, A row-major, B column-major, N(0,1)/sqrt(K):
    every output row against an fp32-accumulating product (torch fp32 on the
    GPU, TF32 off, used only as the checker), and 64 rows against the
    oracle's sequential fp32 sums."""
    import torch
    M = N = K = 8192
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((M, K), dtype=np.float32) / np.sqrt(K)).astype(np.float16)
    Bt = (rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)).astype(np.float16)
    got = hx.gemm_f16_nt(A, Bt)
    fp32_matmul_ieee()
    At = torch.from_numpy(A).cuda().float()
    Btt = torch.from_numpy(Bt).cuda().float()
    for r0 in range(0, M, 2048):
        ref = (At[r0:r0 + 2048] @ Btt.T).half().cpu().numpy()
        assert_f16_gemm_close(got[r0:r0 + 2048], ref)
    del At, Btt
    rows = np.sort(rng.choice(M, 64, replace=False))
    assert_f16_gemm_close(got[rows], oracle.gemm_f16_nt(A[rows], Bt))


from f16_family import F16_BUNDLES, f16_case  # noqa: E402


@pytest.mark.parametrize("bundle", sorted(F16_BUNDLES))
def test_f16_family_golden(hx, bundle):
    A, B, out, kw = f16_case(golden("f16_family"), bundle)
    assert_f16_gemm_close(hx.gemm_f16_ex(A, B, **kw), out)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (130, 257, 200), (512, 384, 1024), (300, 72, 4096)])
def test_f16_ex_random(hx, oracle, M, N, K):
    """Every post-op against the oracle: residual, bias, relu, leaky and GELU
    on the fp16-rounded sum, scaling; B row-major and transposed."""
    rng = np.random.default_rng(M + 7 * N + K)
    A = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    B = rng.standard_normal((K, N)).astype(np.float16)
    Bt = np.ascontiguousarray(B.T)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    for kw in (dict(act="gelu", preround=True), dict(act="leaky", preround=True, bias=bias),
               dict(act="relu", res=res), dict(preround=True, scale=0.0883883476),
               dict(res=res, bias=bias, act="none")):
        exp = oracle.gemm_f16_ex(A, B, **kw)
        assert_f16_gemm_close(hx.gemm_f16_ex(A, B, **kw), exp)
        assert_f16_gemm_close(hx.gemm_f16_ex(A, Bt, b_transposed=True, **kw), exp)


from test_oracle_golden import i8_callers_calls  # noqa: E402


def test_i8_callers_golden(hx):
    for got, exp in i8_callers_calls(hx, golden("i8_callers")):
        np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (1, 4097, 3000), (129, 257, 130), (300, 520, 1000)])
def test_i8_rq_ex_and_s8u8_random(hx, oracle, M, N, K):
    """ReLU-before-requant GEMM (both B layouts, with and without bias) and the
    s8 x u8 HMX field GEMM against the oracle."""
    rng = np.random.default_rng(M + 3 * N + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = rng.integers(-40000, 40000, N).astype(np.int32)
    for kw in (dict(bias=bias, relu=True), dict(relu=False), dict(bias=bias, relu=False)):
        exp = oracle.gemm_i8_rq_ex(A, B, 1234567, 30, 4, **kw)
        np.testing.assert_array_equal(hx.gemm_i8_rq_ex(A, B, 1234567, 30, 4, **kw), exp)
        np.testing.assert_array_equal(
            hx.gemm_i8_rq_ex(A, np.ascontiguousarray(B.T), 1234567, 30, 4, b_transposed=True, **kw), exp)
    Bu = rng.integers(0, 256, (K, N), dtype=np.uint8)
    for store in ("i32", "u16_field", "acc_i32"):
        np.testing.assert_array_equal(hx.gemm_hmx_s8u8(A, Bu, store), oracle.gemm_hmx_s8u8(A, Bu, store))


# ------------------------------------------- CTA-pair vs one-SM GEMM kernel

@pytest.mark.parametrize("M,N,K", [(4096, 2304, 256), (1000, 1800, 520)])
def test_gemm_pair_kernel_matches_single_sm(hx, oracle, monkeypatch, M, N, K):
    """The 256 x 256 CTA-pair kernel (HEXCUDA_GEMM_PAIR=1; the default for
    the fp16 and HMX epilogues when M, N > 128) and the 128-row one-SM kernel
    (HEXCUDA_GEMM_PAIR=0) give identical integer results for every epilogue
    kind, several tiles per pair (accumulator double buffer, ragged edges);
    sampled rows against the oracle."""
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = rng.integers(36, 44, N).astype(np.int32)
    As = rng.integers(-128, 128, (M, K), dtype=np.int8)
    Bt = np.ascontiguousarray(B.T)
    Af = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float16)
    Btf = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float16)

    def run():
        return (hx.gemm_u8s8_pc(A, B, bias, 128, mult, shift, 128),
                hx.gemm_i8_requant(As, B, 1234567, 30, 3),
                hx.gemm_hmx_ex(A, Bt, store="i32", act="relu", bias=bias, b_transposed=True),
                hx.gemm_f16_nt(Af, Btf),
                hx.gemm_f16_nn(Af, np.ascontiguousarray(Btf.T)))

    monkeypatch.setenv("HEXCUDA_GEMM_PAIR", "1")
    pair = run()
    monkeypatch.setenv("HEXCUDA_GEMM_PAIR", "0")
    single = run()
    for p, s in zip(pair[:3], single[:3]):
        np.testing.assert_array_equal(p, s)
    rows = np.sort(rng.choice(M, 16, replace=False))
    np.testing.assert_array_equal(
        pair[0][rows], oracle.gemm_u8s8_pc(A[rows], B, bias, 128, mult, shift, 128))
    np.testing.assert_array_equal(pair[1][rows], oracle.gemm_i8_requant(As[rows], B, 1234567, 30, 3))
    for f in pair[3:]:
        assert_f16_gemm_close(f[rows], oracle.gemm_f16_nt(Af[rows], Btf))


from test_oracle_golden import i8_acc_calls  # noqa: E402


def test_i8_acc_callers_golden(hx):
    for got, exp in i8_acc_calls(hx, golden("i8_acc_callers")):
        np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (129, 257, 130), (300, 520, 1000), (640, 384, 4096)])
def test_i8_acc_random(hx, oracle, M, N, K):
    """Raw-accumulator epilogue (int64 post-ops) on both GEMM kernels,
    signed and unsigned A, every store kind, against the oracle; and the
    requant + int8 residual form."""
    rng = np.random.default_rng(M + N + K)
    A8 = rng.integers(-128, 128, (M, K), dtype=np.int8)
    U8 = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    Bt = np.ascontiguousarray(B.T)
    bias = rng.integers(-2**31, 2**31, N, dtype=np.int64).astype(np.int32)
    res32 = rng.integers(-2**31, 2**31, (M, N), dtype=np.int64).astype(np.int32)
    res8 = rng.integers(-128, 128, (M, N), dtype=np.int8)
    lut8 = rng.integers(-128, 128, 256, dtype=np.int8)
    lut32 = rng.integers(-2**31, 2**31, 256, dtype=np.int64).astype(np.int32)
    cases = [dict(store="i32"), dict(store="i8_sat", act="relu", bias=bias),
             dict(store="u8_sat", res=res8), dict(store="lut_i8", bias=bias, lut=lut8),
             dict(store="lut_i32", act="leaky_shr3", res=res32, lut=lut32),
             dict(store="i8_low", bias=bias, res=res8), dict(store="u16_field", act="relu")]
    for A in (A8, U8):
        for kw in cases:
            exp = oracle.gemm_i8_acc(A, B, **kw)
            np.testing.assert_array_equal(hx.gemm_i8_acc(A, B, **kw), exp, err_msg=str(kw))
            np.testing.assert_array_equal(hx.gemm_i8_acc(A, Bt, b_transposed=True, **kw), exp)
    for mult, shift in ((1 << 30, 44), (-1234567, 20)):
        np.testing.assert_array_equal(hx.gemm_i8_rq_ex(A8, B, mult, shift, 3, bias=bias, res=res8),
                                      oracle.gemm_i8_rq_ex(A8, B, mult, shift, 3, bias=bias, res=res8))


def test_ffn_relu_i8_random(hx, oracle):
    rng = np.random.default_rng(5)
    M, K, V, D = 300, 256, 512, 200
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    W1 = rng.integers(-128, 128, (K, V), dtype=np.int8)
    W2 = rng.integers(-128, 128, (V, D), dtype=np.int8)
    b1 = rng.integers(-50000, 50000, V).astype(np.int32)
    b2 = rng.integers(-50000, 50000, D).astype(np.int32)
    np.testing.assert_array_equal(hx.ffn_relu_i8(A, W1, b1, W2, b2, 1 << 28, 36, 5),
                                  oracle.ffn_relu_i8(A, W1, b1, W2, b2, 1 << 28, 36, 5))


# ------------------------------------------- dot, narrow-GEMM and MLP callers

from test_oracle_golden import dot_calls  # noqa: E402


def test_dot_callers_golden(hx):
    for k, (got, exp) in enumerate(dot_calls(hx, golden("dot_callers"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def _shim(name):
    import ctypes as C
    import subprocess
    from pathlib import Path
    shims = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"
    so = shims / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(shims)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


def test_dot_callers_sdk_shims(hx):
    """The three bundles whose harnesses need the Hexagon SDK, through their
    candidate_kernel shims on the golden cases."""
    import ctypes as C
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    g = golden("dot_callers")
    for n in ("i8_dot_i32_dma", "i16_dot_i32_dma"):
        for t in range(2):
            a, b = g[f"{n}__a{t}"], g[f"{n}__b{t}"]
            out = np.zeros(1, np.int32)
            _shim(n)(p(a), p(b), a.size, p(out))
            np.testing.assert_array_equal(out, g[f"{n}__out{t}"])
    n = "vtcm_stage_matmul_i8"
    A, X = g[n + "__A"], g[n + "__X"]
    out = np.zeros((A.shape[0], X.shape[1]), np.int32)
    _shim(n)(p(A), p(X), p(out), A.shape[0], A.shape[1], X.shape[1])
    np.testing.assert_array_equal(out, g[n + "__out"])


@pytest.mark.parametrize("M,K", [(1, 1), (4097, 8101), (20000, 4096)])
def test_matvec_and_narrow_random(hx, oracle, M, K):
    rng = np.random.default_rng(M + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    x = rng.integers(-128, 128, (1, K), dtype=np.int8)
    np.testing.assert_array_equal(hx.gemm_i8_acc(x, A, b_transposed=True),
                                  oracle.gemm_i8_acc(x, A, b_transposed=True))
    X = rng.integers(-128, 128, (K, 4), dtype=np.int8)
    np.testing.assert_array_equal(hx.gemm_i8_acc(A, X), oracle.gemm_i8_acc(A, X))


def test_outer_product_and_group_dot_random(hx, oracle):
    rng = np.random.default_rng(29)
    a, b = rng.integers(-128, 128, (3000, 1), dtype=np.int8), rng.integers(-128, 128, (1, 5001), dtype=np.int8)
    np.testing.assert_array_equal(hx.gemm_i8_acc(a, b), oracle.gemm_i8_acc(a, b))
    x = rng.integers(-128, 128, (1 << 22) + 44, dtype=np.int8)
    y = rng.integers(-128, 128, (1 << 22) + 44, dtype=np.int8)
    for w in (4, 3, 1, 64):
        np.testing.assert_array_equal(hx.group_dot_i8(x, y, w), oracle.group_dot_i8(x, y, w))
    np.testing.assert_array_equal(hx.group_dot_i8(x[1:], y[1:], 4), oracle.group_dot_i8(x[1:], y[1:], 4))


def test_gate_mul_requant_and_ffn_lut_random(hx, oracle):
    rng = np.random.default_rng(31)
    n = (1 << 22) + 3
    gate, up = rng.integers(-128, 128, n, dtype=np.int8), rng.integers(-128, 128, n, dtype=np.int8)
    lut = rng.integers(-128, 128, 256, dtype=np.int8)
    for mult, shift in ((3, 7), (5, 0), (-(1 << 20), 27), (2**31 - 1, 63), (1 << 30, 40)):
        np.testing.assert_array_equal(hx.gate_mul_requant_i8(gate, up, lut, mult, shift),
                                      oracle.gate_mul_requant_i8(gate, up, lut, mult, shift))
    M, K, V, D = 300, 256, 512, 200
    A = rng.integers(-8, 9, (M, K), dtype=np.int8)
    W1 = rng.integers(-8, 9, (K, V), dtype=np.int8)
    W2 = rng.integers(-128, 128, (V, D), dtype=np.int8)
    b1 = rng.integers(-300, 300, V).astype(np.int32)
    b2 = rng.integers(-50000, 50000, D).astype(np.int32)
    np.testing.assert_array_equal(hx.ffn_lut_i8(A, W1, b1, lut, W2, b2, 1 << 28, 36, 5),
                                  oracle.ffn_lut_i8(A, W1, b1, lut, W2, b2, 1 << 28, 36, 5))


# ---------------------------------------------------------------- int16 GEMM

def test_i16_gemm_golden_and_shim(hx):
    import ctypes as C
    g = golden("affine")
    fn = _shim("i16_gemm")
    for t in range(2):
        A, B, exp = g[f"i16_gemm__A{t}"], g[f"i16_gemm__B{t}"], g[f"i16_gemm__out{t}"]
        np.testing.assert_array_equal(hx.gemm_i16(A, B), exp)
        out = np.zeros_like(exp)
        p = lambda a: a.ctypes.data_as(C.c_void_p)
        fn(p(A), p(B), p(out), A.shape[0], B.shape[1], A.shape[1])
        np.testing.assert_array_equal(out, exp)


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (129, 257, 130), (512, 384, 4099), (1000, 70, 33)])
def test_i16_gemm_random(hx, oracle, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-32768, 32768, (M, K)).astype(np.int16)
    B = rng.integers(-32768, 32768, (K, N)).astype(np.int16)
    np.testing.assert_array_equal(hx.gemm_i16(A, B), oracle.gemm_i16(A, B))
    ext = np.full((M, K), -32768, np.int16), np.full((K, N), 32767, np.int16)
    np.testing.assert_array_equal(hx.gemm_i16(*ext), oracle.gemm_i16(*ext))


# --------------------------------------------------- mixer blocks, RNN cell

from test_oracle_golden import MIX_SETS, mixer_calls  # noqa: E402


def test_mixers_golden_and_shims(hx):
    import ctypes as C
    g = golden("mixers")
    for k, (got, exp) in enumerate(mixer_calls(hx, g)):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    cm, tm, rnn = _shim("i8_channel_mix_block"), _shim("i8_token_mix_block"), _shim("rnn_cell_i8")
    cm.argtypes = [C.c_void_p] * 7 + [C.c_int32, C.c_int, C.c_int32, C.c_int]
    tm.argtypes = [C.c_void_p] * 6 + [C.c_int32, C.c_int, C.c_int32, C.c_int]
    rnn.argtypes = [C.c_void_p] * 6 + [C.c_int, C.c_int, C.c_int32, C.c_int, C.c_int8, C.c_void_p]
    for t, (m1, s1, m2, s2) in enumerate(MIX_SETS):
        out = np.zeros((8, 16), np.int8)
        cm(p(g["X"]), p(g["W1"]), p(g["b1"]), p(g["W2"]), p(g["b2"]), p(g["lut"]), p(out), m1, s1, m2, s2)
        np.testing.assert_array_equal(out, g[f"cmix{t}"])
        tm(p(g["X"]), p(g["Wt"]), p(g["b1"]), p(g["Wt2"]), p(g["bt2"]), p(out), m1, s1, m2, s2)
        np.testing.assert_array_equal(out, g[f"tmix{t}"])
    for t in range(3):
        c = lambda k: g[f"rnn_{k}{t}"]
        mult, shift, zp = (int(v) for v in c("p"))
        H, I = c("Wx").shape
        out = np.zeros(H, np.int8)
        rnn(p(c("Wx")), p(c("Wh")), p(c("b")), p(c("x")), p(c("h")), p(out), H, I, mult, shift, zp, p(g["lut"]))
        np.testing.assert_array_equal(out, c("out"))


def test_mixers_random(hx, oracle):
    rng = np.random.default_rng(43)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    i32 = lambda *sh: rng.integers(-50000, 50000, sh).astype(np.int32)
    lut = s8(256)
    M, K, V, D = 3000, 200, 384, 96
    X, W1, W2 = s8(M, K), s8(V, K), s8(D, V)
    args = (X, W1, i32(V), W2, i32(D), 1 << 12, 20, 77, 14)
    np.testing.assert_array_equal(hx.mix_mlp_i8(*args, lut=lut), oracle.mix_mlp_i8(*args, lut=lut))
    np.testing.assert_array_equal(hx.mix_mlp_i8(*args), oracle.mix_mlp_i8(*args))
    T, Cc, DM = 196, 512, 256
    X, W, W2 = s8(T, Cc), s8(DM, T), s8(T, DM)
    args = (X, W, i32(DM), W2, i32(T), 1 << 12, 19, 99, 14)
    np.testing.assert_array_equal(hx.token_mix_i8(*args), oracle.token_mix_i8(*args))
    for H, I in ((1, 1), (1000, 300), (64, 0)):
        Wx, Wh, x, h = s8(H, I), s8(H, H), s8(I), s8(H)
        args = (Wx, Wh, i32(H), x, h, 1 << 14, 22, 9, lut)
        np.testing.assert_array_equal(hx.rnn_cell_i8(*args), oracle.rnn_cell_i8(*args))


# ------------------------------------------------ HMX-convention convolution

@pytest.mark.parametrize("c_in,ih,iw,c_out,kh,kw,stride", [(8, 10, 10, 32, 3, 3, 1), (3, 31, 17, 40, 5, 3, 2),
                                                          (16, 1, 68, 64, 1, 5, 1), (64, 56, 56, 128, 3, 3, 1)])
def test_conv2d_hmx_random(hx, oracle, c_in, ih, iw, c_out, kh, kw, stride):
    rng = np.random.default_rng(c_in * ih + c_out)
    x = rng.integers(0, 256, (c_in, ih, iw), dtype=np.uint8)
    W = rng.integers(-128, 128, (c_out, c_in, kh, kw), dtype=np.int8)
    bias = rng.integers(-3000, 3000, c_out).astype(np.int32)
    for kw_ in (dict(), dict(bias=bias, store="i32", act="relu"), dict(bias=bias, store="i8_sat")):
        np.testing.assert_array_equal(hx.conv2d_hmx(x, W, stride=stride, **kw_),
                                      oracle.conv2d_hmx(x, W, stride=stride, **kw_), err_msg=str(kw_))
