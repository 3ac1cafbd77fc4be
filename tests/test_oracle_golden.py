"""The CPU oracle (oracle/hexoracle.c) reproduces the reference's own outputs.

Every fixture in tests/golden/ holds inputs regenerated from a corpus
harness recipe (or the benchmark value distributions) and the output of the
reference's scalar reference.c on them (tests/golden/make_golden.py).  The
oracle follows the same arithmetic and accumulation order, so it must match
bit for bit -- integer and floating point alike.
"""
import numpy as np
import pytest

from conftest import golden


def test_i8_gemm_requant_harness(oracle):
    g = golden("i8_gemm_requant_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = oracle.gemm_i8_requant(A, B, int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_i8_gemm_requant_256(oracle):
    g = golden("i8_gemm_requant_256")
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = oracle.gemm_i8_requant(g["A"], g["B"], int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out, g["out"][p])


def test_i8_gemm_requant_256_non_degenerate():
    # the benchmark's own requant (mult ~2^30, shift 8..15) saturates almost
    # everywhere; the fixture's sweep must exercise rounding on real values
    g = golden("i8_gemm_requant_256")
    sat = np.mean(np.abs(g["out"][0].astype(int)) >= 127)
    assert sat > 0.95
    mid = g["out"][1:6]
    assert np.mean(np.abs(mid.astype(int)) < 100) > 0.5


def test_i8_gemm_bias_requant_harness(oracle):
    g = golden("i8_gemm_bias_requant_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = oracle.gemm_i8_bias_requant(A, B, g["bias"], int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_gemm_tile_zp_i8_harness(oracle):
    g = golden("gemm_tile_zp_i8_harness")
    M, N, K = g["dims"]
    A, B = g["A"].reshape(M, K), g["B"].reshape(K, N)
    for p, (zpa, mult, shift) in enumerate(g["params"]):
        out = oracle.gemm_i8_zp(A, B, int(zpa), int(mult), int(shift))
        np.testing.assert_array_equal(out.ravel(), g["out"][p])


def test_requant_per_channel_harness(oracle):
    g = golden("requant_per_channel_harness")
    R, Cc = g["dims"]
    a = g["a"].reshape(R, Cc)
    for k in range(len(g["zp"])):
        out = oracle.requant_per_channel(a, g["mult"][k], g["shift"][k], int(g["zp"][k]))
        np.testing.assert_array_equal(out.ravel(), g["out"][k])


def requantize_input():
    n = 262144
    i = np.arange(n, dtype=np.int64)
    a = (((i * 2731 + 5) & 0xFFFF) - 32768).astype(np.int32)
    a[:6] = [32767, -32768, 0, 6400, 13000, -13000]
    return a


def test_requantize_i32_u8_harness(oracle):
    g = golden("requantize_i32_u8_harness")
    a = requantize_input()
    for p, (mult, shift, zp) in enumerate(g["params"]):
        out = oracle.requantize_i32_u8(a, int(mult), int(shift), int(zp))
        np.testing.assert_array_equal(out, g["out"][p])


def test_gemm_u8s8_pc_small(oracle):
    g = golden("gemm_u8s8_pc_small")
    for c in range(int(g["ncases"])):
        k = lambda s: g[f"c{c}_{s}"]
        out = oracle.gemm_u8s8_pc(k("A"), k("B"), k("bias"), int(k("zpa")), k("mult"), k("shift"),
                                  int(k("zp_out")))
        np.testing.assert_array_equal(out, k("out"))


# (fixture tag, out_kind, b_transposed) of the six HMX-convention bundles,
# harness cases and wide full-range cases
HMX_CASES = [("requant", 1, False), ("zp", 0, False), ("bias_relu", 2, False), ("i64", 0, False),
             ("deepk", 0, False), ("transposeB", 0, True), ("w_requant", 1, False),
             ("w_zp", 0, False), ("w_bias_relu", 2, False), ("w_deepk", 0, False),
             ("w_transposeB", 0, True)]


def hmx_case(g, tag):
    A, B, out = g[f"{tag}_A"], g[f"{tag}_B"], g[f"{tag}_out"]
    K = int(g[f"{tag}_K"]) if f"{tag}_K" in g else int(round(np.sqrt(A.size)))
    M = A.size // K
    N = out.size // M
    zp = int(g[f"{tag}_zp"]) if f"{tag}_zp" in g else 0
    bias = g[f"{tag}_bias"] if f"{tag}_bias" in g else None
    return A.reshape(M, K), B, out.reshape(M, N), K, N, zp, bias


@pytest.mark.parametrize("tag,kind,bt", HMX_CASES)
def test_hmx_gemm_golden(oracle, tag, kind, bt):
    A, B, out, K, N, zp, bias = hmx_case(golden("hmx_gemm"), tag)
    B = B.reshape((N, K) if bt else (K, N))
    got = oracle.gemm_hmx(A, B, kind, bias, zp, bt)
    np.testing.assert_array_equal(got, out)
    if tag.startswith("w_"):
        # the wide cases leave the 12-bit field: outputs wrap / saturate
        assert len(np.unique(got)) > 50


@pytest.mark.parametrize("name,kind", [("gemm_f16_nt_harness", "nt"), ("gemm_f16_nn_harness", "nn"),
                                       ("attn_av_f16_harness", "nn_av")])
def test_f16_gemm_harness(oracle, name, kind):
    g = golden(name)
    M, N, K = g["dims"]
    if kind == "nt":
        out = oracle.gemm_f16_nt(g["A"].reshape(M, K), g["Bt"].reshape(N, K))
    else:
        out = oracle.gemm_f16_nn(g["A"].reshape(M, K), g["B"].reshape(K, N))
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["out"].view(np.uint16))


@pytest.mark.parametrize("name", ["gemm_f16_nt_256x512", "gemm_f16_nt_192x320"])
def test_f16_gemm_multi_tile(oracle, name):
    g = golden(name)
    out = oracle.gemm_f16_nt(g["A"], g["Bt"])
    np.testing.assert_array_equal(out.view(np.uint16), g["out"].view(np.uint16))


@pytest.mark.parametrize("name", ["flash_attn_tile_harness", "flash_attn_256x64x64",
                                  "flash_attn_200x48x128"])
def test_flash_attention(oracle, name):
    g = golden(name)
    Q, K, V = g["Q"], g["K"], g["V"]
    if "dims" in g:
        SQ, SK, DH = g["dims"]
        Q, K, V = Q.reshape(SQ, DH), K.reshape(SK, DH), V.reshape(SK, DH)
    out = oracle.attn_f16(Q, K, V, 0.125, False)
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["O"].ravel().view(np.uint16))


def test_online_softmax_step(oracle):
    g = golden("online_softmax_step_harness")
    for c in range(3):
        st = g[f"c{c}_state_in"]
        m, s, acc = oracle.online_softmax_step_f16(g[f"c{c}_scores"],
                                                   g[f"c{c}_V"].reshape(24, 48), st[0], st[1],
                                                   st[2:])
        got = np.concatenate([[m, s], acc]).astype(np.float16)
        np.testing.assert_array_equal(got.view(np.uint16), g[f"c{c}_state_out"].view(np.uint16))


@pytest.mark.parametrize("name", ["softmax_f16_harness", "softmax_f16_96x256"])
def test_softmax_f16(oracle, name):
    g = golden(name)
    x = g["x"].reshape(-1, 256)
    out = oracle.softmax(x)
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["out"].ravel().view(np.uint16))


def test_layernorm_f16(oracle):
    g = golden("layernorm_f16_harness")
    out = oracle.layernorm(g["x"].reshape(1, -1), g["gamma"], g["beta"], 1e-3)
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["out"].view(np.uint16))


def test_rmsnorm_f16(oracle):
    g = golden("rmsnorm_f16_harness")
    out = oracle.rmsnorm(g["x"].reshape(1, -1), g["gamma"], 1e-3)
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["out"].view(np.uint16))


def test_rowsum_mined_golden(oracle):
    # kernels/mined/fp32_sum: torch-computed golden, accumulation-aware tolerance
    g = golden("rowsum_fp32_mined")
    out = oracle.rowreduce(g["x"].reshape(1, -1), 0)
    e = float(g["out"][0])
    tol = 1e-4 + 1e-3 * abs(e) + float(g["knu"][0]) * float(np.abs(g["x"]).sum())
    assert abs(float(out[0]) - e) <= tol


def test_fp32_restatements_match_fp16_reference_formula(oracle):
    # The fp32 softmax / layernorm used by the 65536 x 4096 benchmark are the
    # fp16 references' formulas with fp32 storage: on inputs exactly
    # representable in fp16, rounding the fp32 oracle's result to fp16 must give
    # the fp16 reference's golden output.
    g = golden("softmax_f16_96x256")
    x32 = g["x"].astype(np.float32)
    out = oracle.softmax(x32).astype(np.float16)
    np.testing.assert_array_equal(out.view(np.uint16), g["out"].view(np.uint16))
    g = golden("layernorm_f16_harness")
    out = oracle.layernorm(g["x"].astype(np.float32).reshape(1, -1), g["gamma"].astype(np.float32),
                           g["beta"].astype(np.float32), 1e-3).astype(np.float16)
    np.testing.assert_array_equal(out.ravel().view(np.uint16), g["out"].view(np.uint16))


from hmx_family import BUNDLES as HMX_FAMILY, golden_case  # noqa: E402


@pytest.mark.parametrize("bundle", sorted(HMX_FAMILY))
def test_hmx_family_golden(oracle, bundle):
    """The generalised HMX epilogue (bias, residual, activation, store kind,
    column-major) against each bundle's own reference.c."""
    A, B, out, kw = golden_case(golden("hmx_family"), bundle)
    np.testing.assert_array_equal(oracle.gemm_hmx_ex(A, B, **kw), out)


from requant_family import RQ_BUNDLES, case_arrays, ew_kwargs  # noqa: E402

RQ_CASES = [(b, c) for b in sorted(RQ_BUNDLES) for c in ("c0", "c1", "c2")
            if c != "c2" or "mult" in RQ_BUNDLES[b][0]]


@pytest.mark.parametrize("bundle,case", RQ_CASES)
def test_requant_family_golden(oracle, bundle, case):
    arr = case_arrays(golden("requant_family"), bundle, case)
    a = arr["a8"] if "a8" in arr else arr["a32"]
    np.testing.assert_array_equal(oracle.requant_ew(a, **ew_kwargs(bundle, arr)), arr["out"])


def test_epilogue_bias_relu_golden(oracle):
    g = golden("requant_family")
    np.testing.assert_array_equal(
        oracle.epilogue_bias_i32(g["epilogue_bias_i32__acc"], g["epilogue_bias_i32__bias"]),
        g["epilogue_bias_i32__out"])
    np.testing.assert_array_equal(oracle.relu_i8(g["epilogue_relu_i8__x"]), g["epilogue_relu_i8__out"])


def test_int8_attention_hmx_golden(oracle):
    g = golden("int8_attention_hmx")
    S, D = g["qkt_SD"]
    np.testing.assert_array_equal(
        oracle.gemm_hmx_ex(g["qkt_Q"].reshape(S, D), g["qkt_K"].reshape(S, D), "u16_field",
                           b_transposed=True), g["qkt_out"].reshape(S, S))
    np.testing.assert_array_equal(
        oracle.gemm_hmx_ex(g["av_P"].reshape(S, S), g["av_V"].reshape(S, D), "u16_field"),
        g["av_out"].reshape(S, D))
    S, D = g["qkav_SD"]
    np.testing.assert_array_equal(
        oracle.attn_qkt_av_hmx(g["qkav_Q"].reshape(S, D), g["qkav_K"].reshape(S, D),
                               g["qkav_V"].reshape(S, D)), g["qkav_out"].reshape(S, D))
    Q, K = g["gqa_Q"].reshape(2, 64, 64), g["gqa_K"].reshape(64, 64)
    for hq in range(2):
        np.testing.assert_array_equal(oracle.gemm_hmx_ex(Q[hq], K, "u16_field", b_transposed=True),
                                      g["gqa_out"].reshape(2, 64, 64)[hq])


def blocks_calls(impl, g):
    """(result, expected) of the five int8 LUT-attention blocks' golden cases
    computed through `impl` (the oracle or the GPU ops module)."""
    lut = g["exp_lut"]
    yield (impl.attn_lut_i8(0 if impl.__name__.endswith("oracle") else "requant", g["gqa_Q"],
                            g["gqa_K"], g["gqa_V"], lut, scale_mult=1 << 30, scale_shift=41,
                            av_mult=1 << 30, av_shift=41), g["gqa_out"])
    hmx = 1 if impl.__name__.endswith("oracle") else "hmx"
    rope = 2 if impl.__name__.endswith("oracle") else "hmx_rope"
    yield (impl.attn_lut_i8(hmx, g["blk_Q"][None], g["blk_K"][None], g["blk_V"][None], lut)[0],
           g["blk_out"])
    yield (impl.attn_lut_i8(hmx, g["gblk_Q"], g["gblk_K"], g["gblk_V"], lut), g["gblk_out"])
    yield (impl.attn_lut_i8(rope, g["rope_Q"][None], g["rope_K"][None], g["rope_V"][None], lut,
                            g["rope_cos"], g["rope_sin"], 6)[0], g["rope_out"])
    yield (impl.decoder_block_i8(g["dec_X"], g["dec_W1"], g["dec_b1"], g["dec_act"], g["dec_W2"],
                                 g["dec_b2"], lut), g["dec_out"])


def test_int8_attention_blocks_golden(oracle):
    for got, exp in blocks_calls(oracle, golden("int8_attention_blocks")):
        np.testing.assert_array_equal(got, exp)


from f16_family import F16_BUNDLES, f16_case  # noqa: E402


@pytest.mark.parametrize("bundle", sorted(F16_BUNDLES))
def test_f16_family_golden(oracle, bundle):
    """The oracle's fp16 post-op GEMM reproduces each bundle's reference.c
    (same fp32 accumulation order, same libm tanh) bit for bit."""
    A, B, out, kw = f16_case(golden("f16_family"), bundle)
    np.testing.assert_array_equal(oracle.gemm_f16_ex(A, B, **kw).view(np.uint16), out.view(np.uint16))


def i8_callers_calls(impl, g):
    """(result, expected) of the int8 GEMM callers' golden cases through
    `impl` (the oracle or the GPU ops module)."""
    yield (impl.gemm_i8_rq_ex(g["gbr_A"], g["gbr_B"], 1 << 30, 38, 3, bias=g["gbr_bias"], relu=True),
           g["gbr_out"])
    x = g["mv_x"][None]
    yield (impl.gemm_i8_rq_ex(x, g["mv_A"], 1 << 30, 38, -2, bias=g["mv_bias"], relu=True,
                              b_transposed=True)[0], g["i8_linear_relu_requant_out"])
    yield (impl.gemm_i8_rq_ex(x, g["mv_A"], 1 << 30, 38, -2, bias=g["mv_bias"], b_transposed=True)[0],
           g["i8_matvec_bias_requant_out"])
    yield (impl.gemm_hmx_ex(g["c11_In"], g["c11_W"], "i32", bias=g["c11_bias"], b_transposed=True),
           g["c11_out"])
    yield (impl.gemm_hmx_ex(g["tbr_A"], g["tbr_B"], "u8_sat", "relu", bias=g["tbr_bias"]), g["tbr_out"])
    for name in ("i8_conv2d_1x1_hmx", "i8_pointwise_conv_hmx"):
        yield impl.gemm_hmx_s8u8(g[name + "_W"], g[name + "_in"], "u16_field"), g[name + "_out"]


def test_i8_callers_golden(oracle):
    for got, exp in i8_callers_calls(oracle, golden("i8_callers")):
        np.testing.assert_array_equal(got, exp)


from reduce_family import golden_case as rd_case, golden_cases as rd_cases, library_call  # noqa: E402

RD_CASES = rd_cases(golden("reduce_family"))


@pytest.mark.parametrize("bundle,case", RD_CASES)
def test_reduce_family_golden(oracle, bundle, case):
    """The oracle's integer reductions, elementwise max / min, group sums,
    prefix max and head-group reduce reproduce each bundle's reference.c."""
    arr = rd_case(golden("reduce_family"), bundle, case)
    np.testing.assert_array_equal(library_call(oracle, bundle, arr), arr["out"])


def test_reduce_family_covers_every_bundle():
    from reduce_family import RD_BUNDLES
    assert {b for b, _ in RD_CASES} == set(RD_BUNDLES)


def i8_acc_calls(impl, g):
    """(result, expected) of the raw-accumulator int8 GEMM callers, the
    requant + residual GEMM and the two-layer FFN (golden i8_acc_callers)
    through `impl` (the oracle or the GPU ops module)."""
    yield impl.gemm_i8_acc(g["gemm_tile_i8__A"], g["gemm_tile_i8__B"], b_transposed=True), g["gemm_tile_i8__out"]
    for name in ("gemm_tile_deepk_i8", "i8_gemm_tile"):
        yield impl.gemm_i8_acc(g[name + "__A"], g[name + "__B"]), g[name + "__out"]
    yield (impl.gemm_i8_acc(g["i8_gemm_bias__A"], g["i8_gemm_bias__B"], bias=g["i8_gemm_bias__bias"]),
           g["i8_gemm_bias__out"])
    A, B, bias = g["i8_batch_matmul__A"], g["i8_batch_matmul__B"], g["i8_batch_matmul_bias__bias"]
    yield np.stack([impl.gemm_i8_acc(A[b], B[b]) for b in range(4)]), g["i8_batch_matmul__out"]
    yield (np.stack([impl.gemm_i8_acc(A[b], B[b], bias=bias[b]) for b in range(4)]),
           g["i8_batch_matmul_bias__out"])
    n = "gemm_tile_bias_relu_i8"
    yield (impl.gemm_i8_acc(g[n + "__A"], g[n + "__B"], "i8_sat", "relu", bias=g[n + "__bias"],
                            b_transposed=True), g[n + "__out"])
    lut = g["gelu_lut"]
    n = "gemm_bias_gelu"
    yield (impl.gemm_i8_acc(g[n + "__A"], g[n + "__B"], "lut_i8", bias=g[n + "__bias"], lut=lut),
           g[n + "__out"])
    yield impl.gemm_i8_acc(g[n + "__A"], g[n + "__B"], "lut_i8", lut=lut), g["i8_gemm_gelu_lut__out"]
    n = "ffn_up_gelu_i8"
    yield (impl.gemm_i8_acc(g[n + "__A"], g[n + "__B"], "lut_i8", bias=g[n + "__bias"], lut=lut,
                            b_transposed=True), g[n + "__out"])
    n = "matmul_residual_add_i8"
    yield (impl.gemm_i8_rq_ex(g[n + "__A"], g[n + "__B"], 1 << 30, 42, 0, res=g[n + "__res"]),
           g[n + "__out"])
    n = "ffn_relu_block"
    yield (impl.ffn_relu_i8(g[n + "__A"], g[n + "__W1"], g[n + "__b1"], g[n + "__W2"], g[n + "__b2"],
                            1 << 24, 30, -3), g[n + "__out"])


def test_i8_acc_callers_golden(oracle):
    for got, exp in i8_acc_calls(oracle, golden("i8_acc_callers")):
        np.testing.assert_array_equal(got, exp)


def dot_calls(impl, g):
    """(result, expected) of the matrix-vector, dot-product, narrow-GEMM,
    outer-product, FFN-down, table-MLP and SiLU-gate bundles (golden
    dot_callers) through `impl` (the oracle or the GPU ops module)."""
    c = lambda n, k: g[f"{n}__{k}"]
    for t in range(2):
        x = c("i8_matvec", f"x{t}")
        yield (impl.gemm_i8_acc(x[None, :], c("i8_matvec", f"A{t}"), b_transposed=True)[0],
               c("i8_matvec", f"out{t}"))
    for t, (mult, shift) in enumerate(((1 << 10, 25), (-7, 17), (3, 0))):
        yield (impl.gemm_i8_rq_ex(c("ffn_down_i8", "A"), c("ffn_down_i8", "B"), mult, shift, 0,
                                  bias=c("ffn_down_i8", "bias"), b_transposed=True),
               c("ffn_down_i8", f"out{t}"))
    for n in ("i8_dot_i32_dma", "i16_dot_i32_dma"):
        for t in range(2):
            yield (np.array([impl.reduce_int(c(n, f"a{t}"), "dot", c(n, f"b{t}"))], np.int32),
                   c(n, f"out{t}"))
    for t in range(2):
        n = "hvx_vrmpy_i8_dot"
        yield impl.group_dot_i8(c(n, f"a{t}"), c(n, f"b{t}")), c(n, f"out{t}")
    n = "vtcm_stage_matmul_i8"
    yield impl.gemm_i8_acc(c(n, "A"), c(n, "X")), c(n, "out")
    for t in range(2):
        n = "i8_outer_product"
        yield impl.gemm_i8_acc(c(n, f"a{t}")[:, None], c(n, f"b{t}")[None, :]), c(n, f"out{t}")
    n = "mlp_block"
    for t, (mult, shift, zp) in enumerate(((3, 10, 0), (7, 11, -3))):
        yield (impl.ffn_lut_i8(c(n, "A"), c(n, "W1"), c(n, "b1"), c(n, "lut"), c(n, "W2"), c(n, "b2"),
                               mult, shift, zp), c(n, f"out{t}"))
    n = "mlp_gate_silu_i8"
    for t, (mult, shift) in enumerate(((3, 7), (5, 3), (1 << 20, 27))):
        yield (impl.gate_mul_requant_i8(c(n, f"gate{t}"), c(n, f"up{t}"), c(n, "lut"), mult, shift),
               c(n, f"out{t}"))


def test_dot_callers_golden(oracle):
    for k, (got, exp) in enumerate(dot_calls(oracle, golden("dot_callers"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def sparse_attn_calls(impl, g):
    """(result, expected) of i8_sparse_attn_block's golden cases through
    `impl` (the oracle or the GPU ops module)."""
    t = 0
    while f"out{t}" in g:
        w, sm, ss, am, ash = (int(v) for v in g[f"params{t}"])
        yield (impl.attn_lut_i8_window(g[f"Q{t}"], g[f"K{t}"], g[f"V{t}"], g[f"lut{t}"], w, sm, ss, am,
                                       ash), g[f"out{t}"])
        t += 1


def test_sparse_attn_golden(oracle):
    n = 0
    for got, exp in sparse_attn_calls(oracle, golden("sparse_attn")):
        np.testing.assert_array_equal(got, exp)
        n += 1
    assert n == 8


def cache_rope_calls(impl, g):
    """(result, expected) of kv_cache_update's and rope_pair_fp16's golden
    cases through `impl` (the oracle or the GPU ops module); the caches are
    updated on copies."""
    for t in range(3):
        kc, vc = g[f"kc{t}"].copy(), g[f"vc{t}"].copy()
        kc, vc = impl.kv_cache_update_i8(kc, vc, g[f"kn{t}"], g[f"vn{t}"], int(g[f"pos{t}"]))
        yield kc, g[f"kout{t}"]
        yield vc, g[f"vout{t}"]
    for t in range(2):
        yield impl.rope_pair_f16(g[f"x{t}"], g[f"cos{t}"], g[f"sin{t}"]), g[f"rope{t}"]


def test_cache_rope_golden(oracle):
    for got, exp in cache_rope_calls(oracle, golden("cache_rope")):
        np.testing.assert_array_equal(got.view(np.uint8), exp.view(np.uint8))


def block_calls(impl, g):
    """(result, expected) of i8_ffn_block, i8_ffn_swiglu_block and
    i8_transformer_encoder_block's golden cases through `impl` (the oracle
    or the GPU ops module)."""
    for t in range(2):
        c = lambda k: g[f"ffn_{k}{t}"]
        yield impl.ffn_hmx_i8(c("X"), c("W1"), c("b1"), c("W2"), c("b2"), 8, 3), c("out")
    for t in range(2):
        c = lambda k: g[f"sw_{k}{t}"]
        yield (impl.ffn_swiglu_hmx_i8(c("X"), c("Wg"), c("Wu"), c("Wd"), c("bd"), c("lut"), 2, 2, 10, 8, 3),
               c("out"))
    for t in range(2):
        c = lambda k: g[f"enc_{k}{t}"]
        yield impl.encoder_block_i8(c("X"), c("W1"), c("b1"), c("W2"), c("b2"), c("lut")), c("out")


def test_blocks_golden(oracle):
    for k, (got, exp) in enumerate(block_calls(oracle, golden("blocks"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def affine_calls(impl, g):
    """(result, expected) of the affine requant bundles and the uint8
    extremes (golden affine) through `impl` (the oracle or the GPU ops)."""
    c = lambda k: g[k]
    x8 = c("x8")
    yield (impl.affine_ew(c("rescale_i16_i8_dma__a0"), np.int8, mult=3, shift=4, wrap32=True),
           c("rescale_i16_i8_dma__out0"))
    for t, (zp, scale, shift) in enumerate(((0, 1, 0), (-7, 300, 3), (100, -77777, 11), (-128, 2**22, 31))):
        yield (impl.affine_ew(x8, np.int16, zp_in=zp, mult=scale, shift=shift, round="floor", wrap32=True),
               c(f"dequant_i8_i16_dma__out{t}"))
    yield (impl.affine_ew(c("hmx_requant_store_i8__a0"), np.int8, mult=17, add=8, shift=4, round="floor",
                          wrap32=True), c("hmx_requant_store_i8__out0"))
    for t, bias in enumerate((0, 77, -200, 100000)):
        yield (impl.affine_ew(x8, np.int8, add=bias, round="floor", wrap32=True),
               c(f"i8_add_bias_sat_dma__out{t}"))
    for t, (scale, sh, s) in enumerate(((1, 0, 0), (3, 5, 2), (-1000, 333, 9), (2**31 - 1, -(2**31), 40))):
        yield impl.affine_ew(x8, np.int8, mult=scale, add=sh, shift=s), c(f"i8_element_affine_dma__out{t}")
    u8 = c("u8")
    for t, m in enumerate((u8.size, 1)):
        yield np.array([impl.reduce_int(u8[:m], "max")], np.uint8), c(f"u8_max_dma__out{t}")
        yield np.array([impl.reduce_int(u8[:m], "min")], np.uint8), c(f"u8_min_dma__out{t}")


RELU6_SCALES = (10, 0, 21, 22, 100, -3)


def clamp_calls(impl, g):
    """(result, expected) of the ReLU / clamp bundles and the global pools
    (golden affine) through `impl`, with the shims' parameter mapping."""
    x8, u8 = g["x8"], g["u8"]
    for name in ("i8_relu_dma", "i8_relu_stream_dma"):
        yield impl.affine_ew(x8, np.int8, round="floor", wrap32=True, lo=0, hi=127), g[name + "__out0"]
    for t, scale in enumerate(RELU6_SCALES):
        cap = int(np.int8(np.int32(6 * scale).astype(np.int8)))
        kw = dict(lo=0, hi=cap) if cap >= 0 else dict(mult=-1000, add=cap, lo=cap, hi=0)
        yield impl.affine_ew(x8, np.int8, round="floor", wrap32=True, **kw), g[f"i8_relu6_dma__out{t}"]
    yield impl.affine_ew(u8, np.uint8, round="floor", wrap32=True, lo=64, hi=191), g["u8_clamp_range_dma__out0"]
    yield (impl.affine_ew(u8, np.uint8, zp_in=128, round="floor", wrap32=True, lo=0, hi=255),
           g["dma_double_buffer_relu_u8__out0"])
    for t, m in enumerate((x8.size, 1, 77)):
        yield np.array([impl.reduce_int(x8[:m], "mean")]).astype(np.int8), g[f"i8_global_avgpool_dma__out{t}"]
        yield np.array([impl.reduce_int(u8[:m], "mean")]).astype(np.uint8), g[f"u8_global_avgpool_dma__out{t}"]
        yield np.array([impl.reduce_int(x8[:m], "max")], np.int8), g[f"i8_global_maxpool_dma__out{t}"]
    yield (impl.affine_ew(u8, np.uint8, zp_in=127, mult=255, round="floor", wrap32=True, lo=0, hi=255),
           g["u8_threshold_dma__out0"])
    yield impl.affine_ew(x8, np.int8, mult=1000, round="floor", wrap32=True, lo=-1, hi=1), g["i8_sign_dma__out0"]
    y8 = g["y8"]
    for name, (lo, hi) in (("i8_add_dma", (-128, 127)), ("i8_add_stream_dma", (-128, 127)),
                           ("i8_vadd_dma", (-256, 255))):
        yield impl.requant_ew(x8, y8, pre="add", lo1=lo, hi1=hi, lo2=lo, hi2=hi), g[name + "__out0"]


MIX_SETS = ((3, 7, 5, 8), (1, 4, 2, 5), (1 << 12, 20, 77, 14))


def mixer_calls(impl, g):
    """(result, expected) of the channel / token mixing blocks and the RNN
    cell (golden mixers) through `impl` (the oracle or the GPU ops)."""
    for t, (m1, s1, m2, s2) in enumerate(MIX_SETS):
        yield (impl.mix_mlp_i8(g["X"], g["W1"], g["b1"], g["W2"], g["b2"], m1, s1, m2, s2, lut=g["lut"]),
               g[f"cmix{t}"])
        yield impl.token_mix_i8(g["X"], g["Wt"], g["b1"], g["Wt2"], g["bt2"], m1, s1, m2, s2), g[f"tmix{t}"]
    for t in range(3):
        c = lambda k: g[f"rnn_{k}{t}"]
        mult, shift, zp = (int(v) for v in c("p"))
        yield impl.rnn_cell_i8(c("Wx"), c("Wh"), c("b"), c("x"), c("h"), mult, shift, zp, g["lut"]), c("out")


def test_mixers_golden(oracle):
    for k, (got, exp) in enumerate(mixer_calls(oracle, golden("mixers"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def test_i16_gemm_golden(oracle):
    g = golden("affine")
    for t in range(2):
        np.testing.assert_array_equal(oracle.gemm_i16(g[f"i16_gemm__A{t}"], g[f"i16_gemm__B{t}"]),
                                      g[f"i16_gemm__out{t}"])


def test_affine_golden(oracle):
    for k, (got, exp) in enumerate(clamp_calls(oracle, golden("affine"))):
        np.testing.assert_array_equal(got, exp, err_msg=f"clamp {k}")
    for k, (got, exp) in enumerate(affine_calls(oracle, golden("affine"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))
    g = golden("affine")
    assert g["u8_max_dma__out2"][0] == 0 and g["u8_min_dma__out2"][0] == 255


NORM_MULT = np.array([3, 5, 7, 9, 11, 13, 15, 17, 3, 5, 7, 9, 11, 13, 15, 17], np.int32)
NORM_SHIFT = np.array([2, 3, 4, 5, 3, 4, 5, 6, 2, 3, 4, 5, 3, 4, 5, 6], np.int32)


def int_rows_calls(impl, g):
    """(result, expected) of the attention-tile callers, the table layernorms
    and softmaxes, the int16 requant, the double requant and the GELU FFN
    block (golden int_rows) through `impl` (the oracle or the GPU ops)."""
    c = lambda n, k: g[f"{n}__{k}"]
    yield (impl.gemm_i8_rq_ex(c("attention_qkt_tile", "Q"), c("attention_qkt_tile", "K"), 1 << 20, 26, 0,
                              b_transposed=True), c("attention_qkt_tile", "out"))
    yield (impl.gemm_i8_rq_ex(c("qkt_tile_i8", "Q"), c("qkt_tile_i8", "K"), 1 << 20, 26, 0),
           c("qkt_tile_i8", "out"))
    yield impl.gemm_i8_acc(c("attention_av_tile", "A"), c("attention_av_tile", "V")), c("attention_av_tile", "out")
    yield (impl.gemm_i8_acc(c("av_tile_i8", "A"), c("av_tile_i8", "V"), b_transposed=True),
           c("av_tile_i8", "out"))
    yield impl.requant_i16(c("attention_scale_i16", "raw"), 1 << 20, 30), c("attention_scale_i16", "out")
    lut = g["exp_lut"][:256]
    yield (impl.gemm_softmax_u8(c("i8_gemm_softmax_tile", "A"), c("i8_gemm_softmax_tile", "B"), lut),
           c("i8_gemm_softmax_tile", "out"))
    yield (impl.gemm_softmax_u8(c("matmul_softmax_tile", "Q"), c("matmul_softmax_tile", "K"), lut,
                                b_transposed=True, requant=True, mult=3000, shift=12),
           c("matmul_softmax_tile", "out"))
    inv = g["inv_lut"]
    n = "i8_layernorm_dma"
    yield impl.layernorm_lut_i8(c(n, "x"), c(n, "gamma"), c(n, "beta"), inv), c(n, "out")
    n = "i8_instance_norm"
    yield (impl.layernorm_lut_i8(c(n, "x"), c(n, "gamma"), c(n, "beta"), c(n, "lut"), "per_row"),
           c(n, "out"))
    n = "i8_chunk_norm"
    ch = c(n, "x").size // 7
    got = impl.layernorm_lut_i8(c(n, "x")[:7 * ch].reshape(7, ch), c(n, "gamma")[:7 * ch],
                                c(n, "beta")[:7 * ch], inv, "rowwise").ravel()
    yield got, c(n, "out")[:7 * ch]
    n = "layernorm_residual"
    yield (impl.layernorm_lut_i8(c(n, "x")[None], c(n, "gamma"), c(n, "beta"), inv,
                                 res=c(n, "res")[None])[0], c(n, "out"))
    n = "embedding_layer_norm"
    yield (impl.layernorm_lut_i8(c(n, "table"), c(n, "gamma"), c(n, "beta"), inv, idx=c(n, "idx")),
           c(n, "out"))
    for n, order in (("layernorm_row_i16", 0), ("layernorm_affine_i16", 1)):
        yield impl.layernorm_lut_i16(c(n, "x"), c(n, "gamma"), c(n, "beta"), g["inv_lut16"], order), c(n, "out")
    n = "i8_norm_requant_dma"
    yield impl.norm_requant_i8(c(n, "x"), NORM_MULT, NORM_SHIFT, 5, 4, 0), c(n, "out")
    n = "gelu_ffn_residual"
    yield (impl.gelu_ffn_residual_i8(*(c(n, k) for k in ("x", "W1", "b1", "gelu_lut", "W2", "b2", "x_res",
                                                          "gamma", "beta")), inv), c(n, "out"))


def test_int_rows_golden(oracle):
    for k, (got, exp) in enumerate(int_rows_calls(oracle, golden("int_rows"))):
        np.testing.assert_array_equal(got, exp, err_msg=str(k))


def test_lut_softmax_i16_properties(oracle):
    """vtcm_softmax_row_i16 (its reference needs the Hexagon SDK headers and
    is not built): the restatement's rows are non-negative, the row maximum
    maps to the largest value, and a constant row gives equal values."""
    rng = np.random.default_rng(4)
    lut = np.sort(rng.integers(1, 65536, 256).astype(np.uint16))
    x = rng.integers(-3000, 3000, (20, 300)).astype(np.int16)
    p = oracle.lut_softmax_i16(x, lut)
    assert (p >= 0).all()
    assert (p[np.arange(20), x.argmax(1)] == p.max(1)).all()
    flat = oracle.lut_softmax_i16(np.full((2, 64), 7, np.int16), lut)
    assert (flat == flat[0, 0]).all()


def softmax_rms_calls(impl, g):
    """(result, expected, tolerance) of the softmax / RMS-norm bundles
    (golden softmax_rms); tolerance None = bit-exact, else the fp16 bar."""
    yield impl.lut_softmax_u8(g["x8"], g["exp_lut"]), g["softmax_rowwise__out"], None
    yield impl.lut_softmax_u8(g["x8"], g["exp_lut"], g["recip_lut"]), g["softmax_row_i8__out"], None
    n = "softmax_row_lut_i16"
    yield impl.lut_softmax_i16(g[n + "__x"], g[n + "__lut"]), g[n + "__out"], None
    n = "rmsnorm_residual"
    yield (impl.layernorm_lut_i8(g[n + "__x"][None], g[n + "__gamma"], None, g[n + "__inv"], "rms",
                                 res=g[n + "__res"][None])[0], g[n + "__out"], None)
    n = "rmsnorm_gain_fp16"
    yield impl.rmsnorm_gain_f16(g[n + "__x"], g[n + "__gain"], 1e-3), g[n + "__out"], 1e-2
    yield (impl.rmsnorm_f16(g["rmsnorm_gain_fp16__x"], g["rmsnorm_row_fp16__gamma"], 1e-3),
           g["rmsnorm_row_fp16__out"], 1e-2)


def check_softmax_rms(impl, g):
    for k, (got, exp, tol) in enumerate(softmax_rms_calls(impl, g)):
        if tol is None:
            np.testing.assert_array_equal(got, exp, err_msg=str(k))
        else:
            e = exp.astype(np.float64)
            assert np.all(np.abs(got.astype(np.float64) - e) <= tol * np.abs(e) + 1e-3 * np.abs(e).max()), k


def test_softmax_rms_golden(oracle):
    check_softmax_rms(oracle, golden("softmax_rms"))
