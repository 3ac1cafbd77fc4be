"""int8 attention blocks with the exp-table softmax on the B200 (one fused
kernel per query head), bit-exact against the reference's outputs and the
oracle."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import golden
from test_oracle_golden import blocks_calls

pytestmark = pytest.mark.gpu

SHIMS = Path(__file__).resolve().parent.parent / "hexkernels_b200" / "shims"


def test_blocks_golden(hx):
    for got, exp in blocks_calls(hx, golden("int8_attention_blocks")):
        np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("HQ,HKV,S,D", [(1, 1, 1, 4), (8, 2, 100, 72), (4, 4, 33, 30), (2, 1, 128, 128)])
def test_attn_lut_random(hx, oracle, HQ, HKV, S, D):
    rng = np.random.default_rng(HQ * 1000 + S + D)
    lut = np.round(255 * np.exp((np.arange(256) - 255) / rng.uniform(8, 40))).astype(np.uint8)
    K = rng.integers(-128, 128, (HKV, S, D), dtype=np.int8)
    V = rng.integers(-128, 128, (HKV, S, D), dtype=np.int8)
    Qs = rng.integers(-128, 128, (HQ, S, D), dtype=np.int8)
    Qu = rng.integers(0, 256, (HQ, S, D), dtype=np.uint8)
    kw = dict(scale_mult=1 << 30, scale_shift=40, av_mult=3 << 28, av_shift=40)
    np.testing.assert_array_equal(hx.attn_lut_i8("requant", Qs, K, V, lut, **kw),
                                  oracle.attn_lut_i8(0, Qs, K, V, lut, **kw))
    np.testing.assert_array_equal(hx.attn_lut_i8("hmx", Qu, K, V, lut),
                                  oracle.attn_lut_i8(1, Qu, K, V, lut))
    if D % 2 == 0:
        cs = rng.integers(-64, 65, (S, D // 2)).astype(np.int8)
        sn = rng.integers(-64, 65, (S, D // 2)).astype(np.int8)
        np.testing.assert_array_equal(hx.attn_lut_i8("hmx_rope", Qu, K, V, lut, cs, sn, 5),
                                      oracle.attn_lut_i8(2, Qu, K, V, lut, cs, sn, 5))


@pytest.mark.parametrize("S,D,F", [(1, 4, 4), (60, 96, 200), (33, 30, 70)])
def test_decoder_block_random(hx, oracle, S, D, F):
    rng = np.random.default_rng(S + D + F)
    lut = np.round(255 * np.exp((np.arange(256) - 255) / 24.0)).astype(np.uint8)
    X = rng.integers(0, 64, (S, D), dtype=np.uint8)
    W1 = rng.integers(-128, 128, (D, F), dtype=np.int8)
    W2 = rng.integers(-128, 128, (F, D), dtype=np.int8)
    b1 = rng.integers(-300, 300, F).astype(np.int32)
    b2 = rng.integers(-60, 60, D).astype(np.int32)
    act = rng.integers(-128, 128, 256).astype(np.int8)
    np.testing.assert_array_equal(hx.decoder_block_i8(X, W1, b1, act, W2, b2, lut),
                                  oracle.decoder_block_i8(X, W1, b1, act, W2, b2, lut))


def shim(name):
    so = SHIMS / f"libcand_{name}.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(SHIMS)], check=True)
    fn = C.CDLL(str(so)).candidate_kernel
    fn.restype = None
    return fn


def test_block_shims(hx):
    g = golden("int8_attention_blocks")
    p = lambda a: np.ascontiguousarray(a).ctypes.data_as(C.c_void_p)
    lut = g["exp_lut"]
    o = np.zeros_like(g["gqa_out"])
    shim("gqa_attention")(p(g["gqa_Q"]), p(g["gqa_K"]), p(g["gqa_V"]), p(lut), p(o), C.c_int32(1 << 30),
                          41, C.c_int32(1 << 30), 41)
    np.testing.assert_array_equal(o, g["gqa_out"])
    S, D = g["blk_out"].shape
    o = np.zeros_like(g["blk_out"])
    shim("i8_attention_block")(p(g["blk_Q"]), p(g["blk_K"]), p(g["blk_V"]), p(o), S, D, p(lut))
    np.testing.assert_array_equal(o, g["blk_out"])
    o = np.zeros_like(g["gblk_out"])
    shim("i8_gqa_attention_block")(p(g["gblk_Q"]), p(g["gblk_K"]), p(g["gblk_V"]), p(o), p(lut))
    np.testing.assert_array_equal(o, g["gblk_out"])
    S, D = g["rope_out"].shape
    o = np.zeros_like(g["rope_out"])
    shim("i8_rope_attention_block")(p(g["rope_Q"]), p(g["rope_K"]), p(g["rope_V"]), p(g["rope_cos"]),
                                    p(g["rope_sin"]), p(o), S, D, 6, p(lut))
    np.testing.assert_array_equal(o, g["rope_out"])
    S, D = g["dec_out"].shape
    o = np.zeros_like(g["dec_out"])
    shim("i8_decoder_block")(p(g["dec_X"]), p(g["dec_W1"]), p(g["dec_b1"]), p(g["dec_act"]),
                             p(g["dec_W2"]), p(g["dec_b2"]), p(lut), p(o), S, D, g["dec_W1"].shape[1])
    np.testing.assert_array_equal(o, g["dec_out"])
