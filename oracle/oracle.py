"""NumPy wrapper of the CPU oracle (hexoracle.c) -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use
this module, as the checker or the timed CPU baseline.  The product path
(hexkernels_b200) never imports it.  liboracle.so is built on first use with
the oracle Makefile (gcc only).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
P = C.c_void_p
_lib = None
_ref = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        so = HERE / "liboracle.so"
        if not so.exists():
            build()
        _lib = C.CDLL(str(so))
    return _lib


def ref_lib() -> C.CDLL | None:
    """The reference's own scalar code (oracle/_ref/libhexref.so) if built."""
    global _ref
    if _ref is None:
        so = HERE / "_ref" / "libhexref.so"
        if so.exists():
            _ref = C.CDLL(str(so))
    return _ref


def _p(a):
    return a.ctypes.data_as(P)


def nthreads_default() -> int:
    return len(os.sched_getaffinity(0))


# ------------------------------------------------------------------ integer

def gemm_i8_requant(A, B, mult, shift, zp, rows=None):
    A, B = np.ascontiguousarray(A, np.int8), np.ascontiguousarray(B, np.int8)
    (M, K), (_, N) = A.shape, B.shape
    r0, r1 = rows or (0, M)
    out = np.zeros((M, N), np.int8)
    lib().oracle_i8_gemm_requant_rows(_p(A), _p(B), _p(out), M, N, K, C.c_int32(mult),
                                      C.c_int(shift), C.c_int8(zp), r0, r1)
    return out


def gemm_i8_bias_requant(A, B, bias, mult, shift, zp):
    A, B = np.ascontiguousarray(A, np.int8), np.ascontiguousarray(B, np.int8)
    bias = np.ascontiguousarray(bias, np.int32)
    (M, K), (_, N) = A.shape, B.shape
    out = np.zeros((M, N), np.int8)
    lib().oracle_i8_gemm_bias_requant_rows(_p(A), _p(B), _p(bias), _p(out), M, N, K,
                                           C.c_int32(mult), C.c_int(shift), C.c_int8(zp), 0, M)
    return out


def gemm_i8_zp(A, B, zpA, mult, shift):
    A, B = np.ascontiguousarray(A, np.int8), np.ascontiguousarray(B, np.int8)
    (M, K), (_, N) = A.shape, B.shape
    out = np.zeros((M, N), np.int8)
    lib().oracle_gemm_tile_zp_i8_rows(_p(A), _p(B), _p(out), M, N, K, C.c_int32(zpA),
                                      C.c_int32(mult), C.c_int(shift), 0, M)
    return out


def gemm_u8s8_pc(A, B, bias, zpA, mult, shift, zp_out, rows=None):
    A, B = np.ascontiguousarray(A, np.uint8), np.ascontiguousarray(B, np.int8)
    bias = np.ascontiguousarray(bias, np.int32)
    mult, shift = np.ascontiguousarray(mult, np.int32), np.ascontiguousarray(shift, np.int32)
    (M, K), (_, N) = A.shape, B.shape
    r0, r1 = rows or (0, M)
    out = np.zeros((M, N), np.uint8)
    lib().oracle_gemm_u8s8_pc_rows(_p(A), _p(B), _p(bias), _p(out), M, N, K, C.c_int32(zpA),
                                   _p(mult), _p(shift), C.c_uint8(zp_out), r0, r1)
    return out


def gemm_hmx(A, B, out_kind=0, bias=None, zpA=0, b_transposed=False):
    """HMX-convention u8 x s8 GEMM: out_kind 0 int32, 1 int8, 2 uint8 bias-ReLU."""
    A, B = np.ascontiguousarray(A, np.uint8), np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    out = np.zeros((M, N), {0: np.int32, 1: np.int8, 2: np.uint8}[out_kind])
    if out_kind == 2:
        bias = np.ascontiguousarray(bias, np.int32)
    lib().oracle_gemm_hmx_rows(_p(A), _p(B), int(b_transposed),
                               _p(bias) if bias is not None else None, _p(out), M, N, K,
                               C.c_int32(zpA), out_kind, 0, M)
    return out


def gemm_hmx_ex(A, B, store="i32", act="none", bias=None, res=None, lut=None, zpA=0,
                b_transposed=False, col_major=False):
    stores = {"i32": (0, np.int32), "i8_sat": (1, np.int8), "u8_sat": (2, np.uint8),
              "i8_low": (3, np.int8), "u16_field": (4, np.uint16), "lut_i32": (5, np.int32),
              "lut_i8": (6, np.int8), "acc_i32": (7, np.int32)}
    A, B = np.ascontiguousarray(A, np.uint8), np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    kind, dt = stores[store]
    out = np.zeros((N, M) if col_major else (M, N), dt)
    res_kind = 0
    if res is not None:
        res = np.ascontiguousarray(res)
        res_kind = 1 if res.dtype == np.int32 else 2
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.int32)
    if lut is not None:
        lut = np.ascontiguousarray(lut, np.int32 if store == "lut_i32" else np.int8)
    pp = lambda a: _p(a) if a is not None else None
    lib().oracle_gemm_hmx_ex_rows(_p(A), _p(B), int(b_transposed), _p(out), M, N, K,
                                  C.c_int32(zpA), kind, {"none": 0, "relu": 1, "leaky_shr3": 2}[act],
                                  pp(bias), res_kind, pp(res), pp(lut), int(col_major), 0, M)
    return out


def requant_ew(a, b=None, pre="a", pre_c=0, mult=1, shift=0, zp=0, sign_of_a=False,
               lo1=-128, hi1=127, lo2=-128, hi2=127, lut=None, out_dtype=np.int8):
    a = np.ascontiguousarray(a)
    b_kind = 0
    if b is not None:
        b = np.ascontiguousarray(b)
        b_kind = 1 if b.dtype == np.int32 else 2
    if lut is not None:
        lut = np.ascontiguousarray(lut, np.int8)
    out = np.zeros(a.shape, out_dtype)
    lib().oracle_requant_ew(_p(a), int(a.dtype == np.int8), _p(b) if b is not None else None,
                            b_kind, C.c_int64(a.size),
                            {"a": 0, "add": 1, "add_relu": 2, "mul_add": 3}[pre], C.c_int64(pre_c),
                            C.c_int32(mult), shift, zp, int(sign_of_a), lo1, hi1, lo2, hi2,
                            _p(lut) if lut is not None else None, _p(out))
    return out


def epilogue_bias_i32(acc, bias):
    acc, bias = np.ascontiguousarray(acc, np.int32), np.ascontiguousarray(bias, np.int32)
    R, Cc = acc.shape
    out = np.zeros_like(acc)
    lib().oracle_epilogue_bias_i32(_p(acc), _p(bias), _p(out), R, Cc)
    return out


def relu_i8(x):
    x = np.ascontiguousarray(x, np.int8)
    out = np.zeros_like(x)
    lib().oracle_relu_i8(_p(x), _p(out), C.c_int64(x.size))
    return out


def attn_qkt_av_hmx(Q, K, V):
    Q, K, V = (np.ascontiguousarray(Q, np.uint8), np.ascontiguousarray(K, np.int8),
               np.ascontiguousarray(V, np.int8))
    (SQ, D), (SK, _) = Q.shape, K.shape
    out = np.zeros((SQ, D), np.int32)
    lib().oracle_attn_qkt_av_hmx(_p(Q), _p(K), _p(V), _p(out), SQ, SK, D)
    return out


def attn_lut_i8(mode, Q, K, V, exp_lut, cos_lut=None, sin_lut=None, rot_shift=0,
                scale_mult=0, scale_shift=0, av_mult=0, av_shift=0):
    """Q [HQ, S, D], K / V [HKV, S, D]; mode 0 requant (int8 out), 1 HMX, 2 HMX + rotation."""
    Q = np.ascontiguousarray(Q, np.int8 if mode == 0 else np.uint8)
    K, V = np.ascontiguousarray(K, np.int8), np.ascontiguousarray(V, np.int8)
    HQ, S, D = Q.shape
    out = np.zeros(Q.shape, np.int8 if mode == 0 else np.uint16)
    pp = lambda a: _p(np.ascontiguousarray(a)) if a is not None else None
    lib().oracle_attn_lut_i8(mode, _p(Q), _p(K), _p(V), pp(np.asarray(exp_lut, np.uint8)),
                             pp(cos_lut), pp(sin_lut), rot_shift, _p(out), HQ, K.shape[0], S, D,
                             C.c_int32(scale_mult), scale_shift, C.c_int32(av_mult), av_shift)
    return out


def attn_lut_i8_window(Q, K, V, exp_lut, window, scale_mult, scale_shift, av_mult, av_shift):
    """Q / K / V [H, S, D] int8; requant scores outside |i - j| <= window set to -128."""
    Q, K, V = (np.ascontiguousarray(x, np.int8) for x in (Q, K, V))
    H, S, D = Q.shape
    out = np.zeros(Q.shape, np.int8)
    lib().oracle_attn_lut_i8_window(_p(Q), _p(K), _p(V), _p(np.ascontiguousarray(exp_lut, np.uint8)),
                                    _p(out), H, S, D, window, C.c_int32(scale_mult), scale_shift,
                                    C.c_int32(av_mult), av_shift)
    return out


def decoder_block_i8(X, W1, b1, act_lut, W2, b2, exp_lut):
    X = np.ascontiguousarray(X, np.uint8)
    W1, W2 = np.ascontiguousarray(W1, np.int8), np.ascontiguousarray(W2, np.int8)
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    act_lut, exp_lut = np.ascontiguousarray(act_lut, np.int8), np.ascontiguousarray(exp_lut, np.uint8)
    S, D = X.shape
    out = np.zeros((S, D), np.int8)
    lib().oracle_decoder_block_i8(_p(X), _p(W1), _p(b1), _p(act_lut), _p(W2), _p(b2), _p(exp_lut),
                                  _p(out), S, D, W1.shape[1])
    return out


def gemm_f16_ex(A, B, act="none", preround=False, scale=1.0, bias=None, res=None,
                b_transposed=False):
    A, B = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(B, np.float16)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    out = np.zeros((M, N), np.float16)
    pp = lambda a: _p(np.ascontiguousarray(a, np.float16)) if a is not None else None
    keep = [np.ascontiguousarray(x, np.float16) for x in (bias, res) if x is not None]
    lib().oracle_gemm_f16_ex_rows(_p(A), _p(B), int(b_transposed),
                                  _p(keep[0]) if bias is not None else None,
                                  _p(keep[-1]) if res is not None else None, _p(out), M, N, K,
                                  {"none": 0, "relu": 1, "leaky": 2, "gelu": 3, "sigmoid": 4,
                                   "tanh": 5}[act], {False: 0, True: 1, "sum": 1, "acc": 2}[preround],
                                  C.c_float(scale), 0, M)
    return out


def gemm_i8_rq_ex(A, B, mult, shift, zp, bias=None, relu=False, b_transposed=False, res=None):
    A, B = np.ascontiguousarray(A, np.int8), np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    out = np.zeros((M, N), np.int8)
    bias = np.ascontiguousarray(bias, np.int32) if bias is not None else None
    res = np.ascontiguousarray(res, np.int8) if res is not None else None
    lib().oracle_gemm_i8_rq_ex_rows(_p(A), _p(B), int(b_transposed),
                                    _p(bias) if bias is not None else None,
                                    _p(res) if res is not None else None, _p(out), M, N, K,
                                    C.c_int32(mult), shift, zp, int(relu), 0, M)
    return out


HMX_STORE = {"i32": (0, np.int32), "i8_sat": (1, np.int8), "u8_sat": (2, np.uint8),
             "i8_low": (3, np.int8), "u16_field": (4, np.uint16), "lut_i32": (5, np.int32),
             "lut_i8": (6, np.int8), "acc_i32": (7, np.int32)}
HMX_ACT = {"none": 0, "relu": 1, "leaky_shr3": 2}


def gemm_i8_acc(A, B, store="i32", act="none", bias=None, res=None, lut=None, b_transposed=False):
    A = np.ascontiguousarray(A)
    a_signed = int(A.dtype == np.int8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    kind, dt = HMX_STORE[store]
    out = np.zeros((M, N), dt)
    res_kind = 0
    if res is not None:
        res = np.ascontiguousarray(res)
        res_kind = 1 if res.dtype == np.int32 else 2
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.int32)
    if lut is not None:
        lut = np.ascontiguousarray(lut, np.int32 if store == "lut_i32" else np.int8)
    pp = lambda a: _p(a) if a is not None else None
    lib().oracle_gemm_i8_acc_rows(_p(A), a_signed, _p(B), int(b_transposed), pp(bias), pp(res),
                                  res_kind, pp(lut), _p(out), kind, HMX_ACT[act], M, N, K, 0, M)
    return out


def ffn_relu_i8(A, W1, b1, W2, b2, mult, shift, zp):
    A, W1, W2 = (np.ascontiguousarray(x, np.int8) for x in (A, W1, W2))
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    (M, K), (_, V), (_, D) = A.shape, W1.shape, W2.shape
    out = np.zeros((M, D), np.int8)
    lib().oracle_ffn_relu_i8(_p(A), _p(W1), _p(b1), _p(W2), _p(b2), _p(out), M, K, V, D,
                             C.c_int32(mult), shift, zp)
    return out


def ffn_lut_i8(A, W1, b1, act_lut, W2, b2, mult, shift, zp):
    A, W1, W2, act_lut = (np.ascontiguousarray(x, np.int8) for x in (A, W1, W2, act_lut))
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    (M, K), (_, V), (_, D) = A.shape, W1.shape, W2.shape
    out = np.zeros((M, D), np.int8)
    lib().oracle_ffn_lut_i8(_p(A), _p(W1), _p(b1), _p(act_lut), _p(W2), _p(b2), _p(out), M, K, V,
                            D, C.c_int32(mult), shift, zp)
    return out


def gemm_hmx_s8u8(A, B, store="i32"):
    A, B = np.ascontiguousarray(A, np.int8), np.ascontiguousarray(B, np.uint8)
    M, K = A.shape
    N = B.shape[1]
    kind, dt = {"i32": (0, np.int32), "u16_field": (4, np.uint16), "acc_i32": (7, np.int32)}[store]
    out = np.zeros((M, N), dt)
    lib().oracle_gemm_hmx_s8u8_rows(_p(A), _p(B), _p(out), kind, M, N, K, 0, M)
    return out


def requant_per_channel(a, mult, shift, zp):
    a = np.ascontiguousarray(a, np.int32)
    R, Cc = a.shape
    mult, shift = np.ascontiguousarray(mult, np.int32), np.ascontiguousarray(shift, np.int32)
    out = np.zeros((R, Cc), np.int8)
    lib().oracle_requant_per_channel(_p(a), _p(out), R, Cc, _p(mult), _p(shift), C.c_int8(zp))
    return out


def requantize_i32_u8(a, mult, shift, zp):
    a = np.ascontiguousarray(a, np.int32)
    out = np.zeros(a.shape, np.uint8)
    lib().oracle_requantize_i32_u8(_p(a), _p(out), C.c_int64(a.size), C.c_int32(mult),
                                   C.c_int(shift), C.c_uint8(zp))
    return out


# --------------------------------------------------------------------- fp16

def gemm_f16_nt(A, Bt, rows=None):
    A, Bt = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(Bt, np.float16)
    (M, K), (N, _) = A.shape, Bt.shape
    r0, r1 = rows or (0, M)
    out = np.zeros((M, N), np.float16)
    lib().oracle_gemm_f16_nt_rows(_p(A), _p(Bt), _p(out), M, N, K, r0, r1)
    return out


def gemm_f16_nn(A, B):
    A, B = np.ascontiguousarray(A, np.float16), np.ascontiguousarray(B, np.float16)
    (M, K), (_, N) = A.shape, B.shape
    out = np.zeros((M, N), np.float16)
    lib().oracle_gemm_f16_nn_rows(_p(A), _p(B), _p(out), M, N, K, 0, M)
    return out


def attn_f16(Q, K, V, scale, causal, heads=None):
    Q, K, V = (np.ascontiguousarray(t, np.float16) for t in (Q, K, V))
    SQ, D = Q.shape[-2:]
    SK = K.shape[-2]
    BH = int(np.prod(Q.shape[:-2])) if Q.ndim > 2 else 1
    h0, h1 = heads or (0, BH)
    O = np.zeros(Q.shape, np.float16)
    lib().oracle_attn_f16_heads(_p(Q), _p(K), _p(V), _p(O), BH, SQ, SK, D, C.c_float(scale),
                                int(bool(causal)), h0, h1)
    return O


def online_softmax_step_f16(scores, V, running_max, running_sum, acc):
    scores, V = np.ascontiguousarray(scores, np.float16), np.ascontiguousarray(V, np.float16)
    acc = np.array(acc, np.float16, copy=True)
    BLK, D = V.shape
    m = np.array([running_max], np.float16)
    s = np.array([running_sum], np.float16)
    lib().oracle_online_softmax_step_f16(_p(scores), _p(V), _p(m), _p(s), _p(acc), BLK, D)
    return m[0], s[0], acc


# --------------------------------------------------------------------- rows

def softmax(x):
    x = np.ascontiguousarray(x)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros_like(x)
    if x.dtype == np.float32:
        lib().oracle_softmax_f32_rows(_p(x), _p(out), R, Cc, 0, R)
    else:
        lib().oracle_softmax_f16_rows(_p(x), _p(out), R, Cc, 0, R)
    return out


def layernorm(x, gamma, beta, eps):
    x = np.ascontiguousarray(x)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    gamma, beta = np.ascontiguousarray(gamma, x.dtype), np.ascontiguousarray(beta, x.dtype)
    out = np.zeros_like(x)
    if x.dtype == np.float32:
        lib().oracle_layernorm_f32_rows(_p(x), _p(gamma), _p(beta), _p(out), R, Cc,
                                        C.c_float(eps), 0, R)
    else:
        lib().oracle_layernorm_f16_rows(_p(x), _p(gamma), _p(beta), _p(out), R, Cc,
                                        C.c_float(eps), 0, R)
    return out


def rmsnorm(x, gamma, eps):
    x = np.ascontiguousarray(x)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    gamma = np.ascontiguousarray(gamma, x.dtype)
    out = np.zeros_like(x)
    if x.dtype == np.float32:
        lib().oracle_rmsnorm_f32_rows(_p(x), _p(gamma), _p(out), R, Cc, C.c_float(eps), 0, R)
    else:
        lib().oracle_rmsnorm_f16_rows(_p(x), _p(gamma), _p(out), R, Cc, C.c_float(eps), 0, R)
    return out


def rowreduce(x, op):
    x = np.ascontiguousarray(x, np.float32)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    out = np.zeros(R, np.float32)
    lib().oracle_rowreduce_f32_rows(_p(x), _p(out), R, Cc, op, 0, R)
    return out


# ------------------------------------------------------ threaded (baseline)

class _GemmArgs(C.Structure):
    _fields_ = [("A", P), ("B", P), ("bias", P), ("out", P), ("M", C.c_int), ("N", C.c_int),
                ("K", C.c_int), ("zpA", C.c_int32), ("mult", C.c_int32), ("shift", C.c_int),
                ("zp", C.c_int), ("mult_pc", P), ("shift_pc", P)]


class _AttnArgs(C.Structure):
    _fields_ = [("Q", P), ("K", P), ("V", P), ("O", P), ("BH", C.c_int), ("SQ", C.c_int),
                ("SK", C.c_int), ("D", C.c_int), ("scale", C.c_float), ("causal", C.c_int)]


class _RowsArgs(C.Structure):
    _fields_ = [("x", P), ("gamma", P), ("beta", P), ("out", P), ("R", C.c_int), ("C", C.c_int),
                ("eps", C.c_float), ("op", C.c_int)]


OP_I8_GEMM_REQUANT, OP_GEMM_U8S8_PC, OP_GEMM_F16_NT, OP_ATTN_F16 = 1, 2, 3, 4
OP_SOFTMAX_F32, OP_LAYERNORM_F32, OP_ROWREDUCE_F32 = 5, 6, 7


def parallel(op: int, args: C.Structure, r0: int, r1: int, nthreads: int) -> None:
    rc = lib().oracle_parallel(op, C.byref(args), r0, r1, nthreads)
    if rc:
        raise RuntimeError(f"oracle_parallel failed ({rc})")


def gemm_args(**kw) -> _GemmArgs:
    a = _GemmArgs()
    for k, v in kw.items():
        setattr(a, k, _p(v) if isinstance(v, np.ndarray) else v)
    return a


def attn_args(**kw) -> _AttnArgs:
    a = _AttnArgs()
    for k, v in kw.items():
        setattr(a, k, _p(v) if isinstance(v, np.ndarray) else v)
    return a


def rows_args(**kw) -> _RowsArgs:
    a = _RowsArgs()
    for k, v in kw.items():
        setattr(a, k, _p(v) if isinstance(v, np.ndarray) else v)
    return a


ELEM = {np.dtype(np.int8): 0, np.dtype(np.uint8): 1, np.dtype(np.int16): 2,
        np.dtype(np.int32): 3}
RED_OPS = {"sum": 0, "sum64": 1, "sumsq": 2, "sumsq_diff": 3, "dot": 4, "l1": 5, "absmax": 6,
           "max": 7, "min": 8, "argmax": 9, "argmin": 10, "top1": 11, "mean": 12}


def reduce_int(a, op, b=None):
    a = np.ascontiguousarray(a).ravel()
    if b is not None:
        b = np.ascontiguousarray(b, a.dtype).ravel()
    out = np.zeros(2, np.int64 if op == "sum64" else np.int32)
    lib().oracle_reduce_int(_p(a), _p(b) if b is not None else None, ELEM[a.dtype],
                            C.c_int64(a.size), RED_OPS[op], _p(out))
    return (int(out[0]), int(out[1])) if op == "top1" else int(out[0])


def minmax_ew(a, b=None, c=0, op="max"):
    a = np.ascontiguousarray(a)
    out = np.zeros_like(a)
    lib().oracle_minmax_ew(_p(a), _p(np.ascontiguousarray(b, a.dtype)) if b is not None else None,
                           C.c_int32(int(c)), ELEM[a.dtype], {"max": 0, "min": 1}[op], _p(out),
                           C.c_int64(a.size))
    return out


def group_sum_i8(a, w=4):
    a = np.ascontiguousarray(a, np.int8).ravel()
    g = a.size // w
    out = np.zeros(g, np.int32)
    lib().oracle_group_sum_i8(_p(a), _p(out), C.c_int64(g), w)
    return out


def group_dot_i8(a, b, w=4):
    a = np.ascontiguousarray(a, np.int8).ravel()
    b = np.ascontiguousarray(b, np.int8).ravel()
    g = a.size // w
    out = np.zeros(g, np.int32)
    lib().oracle_group_dot_i8(_p(a), _p(b), _p(out), C.c_int64(g), w)
    return out


def gate_mul_requant_i8(gate, up, lut, mult, shift):
    gate, up = np.ascontiguousarray(gate, np.int8), np.ascontiguousarray(up, np.int8)
    lut = np.ascontiguousarray(lut, np.int8)
    out = np.zeros(gate.shape, np.int8)
    lib().oracle_gate_mul_requant_i8(_p(gate), _p(up), _p(lut), _p(out), C.c_int64(gate.size),
                                     C.c_int32(int(mult)), shift)
    return out


def scan_max_i8(x):
    x = np.ascontiguousarray(x, np.int8).ravel()
    out = np.zeros_like(x)
    lib().oracle_scan_max_i8(_p(x), _p(out), C.c_int64(x.size))
    return out


def head_group_reduce_i8(X, G, mult, shift):
    X = np.ascontiguousarray(X, np.int8)
    H = X.shape[0]
    MN = int(np.prod(X.shape[1:]))
    Y = np.zeros((G,) + X.shape[1:], np.int8)
    lib().oracle_head_group_reduce_i8(_p(X), _p(Y), H, G, C.c_int64(MN), C.c_int32(int(mult)),
                                      shift)
    return Y


LN_AFFINE = {"shared": 0, "rowwise": 1, "per_row": 2, "rms": 3}


def layernorm_lut_i8(x, gamma, beta, inv_lut, affine="shared", res=None, idx=None):
    x = np.ascontiguousarray(x, np.int8)
    W = x.shape[1]
    idx = np.ascontiguousarray(idx, np.int32) if idx is not None else None
    R = idx.size if idx is not None else x.shape[0]
    res = np.ascontiguousarray(res, np.int8) if res is not None else None
    g, lut = np.ascontiguousarray(gamma, np.int8), np.ascontiguousarray(inv_lut, np.uint8)
    b = np.ascontiguousarray(beta, np.int8) if beta is not None else None
    out = np.zeros((R, W), np.int8)
    lib().oracle_layernorm_lut_i8(_p(x), None if idx is None else _p(idx),
                                  None if res is None else _p(res), _p(out), R, W, _p(g),
                                  _p(b) if b is not None else None, _p(lut), LN_AFFINE[affine])
    return out


def layernorm_lut_i16(x, gamma, beta, inv_lut, order=0):
    x = np.ascontiguousarray(x, np.int16)
    R, Cc = x.shape
    out = np.zeros_like(x)
    g, b, lut = (np.ascontiguousarray(gamma, np.int16), np.ascontiguousarray(beta, np.int16),
                 np.ascontiguousarray(inv_lut, np.uint16))
    lib().oracle_layernorm_lut_i16(_p(x), _p(out), R, Cc, _p(g), _p(b), _p(lut), order)
    return out


def lut_softmax_u8(x, exp_lut, recip_lut=None):
    x = np.ascontiguousarray(x, np.int8)
    out = np.zeros(x.shape, np.uint8)
    lut = np.ascontiguousarray(exp_lut, np.uint8)
    rl = np.ascontiguousarray(recip_lut, np.uint16) if recip_lut is not None else None
    lib().oracle_lut_softmax_u8(_p(x), _p(out), x.shape[0], x.shape[1], _p(lut),
                                _p(rl) if rl is not None else None)
    return out


def rmsnorm_gain_f16(x, gain, eps):
    x = np.ascontiguousarray(x, np.float16)
    g = np.ascontiguousarray(gain, np.float16)
    out = np.zeros_like(x)
    lib().oracle_rmsnorm_gain_f16(_p(x), _p(g), _p(out), x.shape[0], x.shape[1], C.c_float(eps))
    return out


def lut_softmax_i16(x, exp_lut):
    x = np.ascontiguousarray(x, np.int16)
    out = np.zeros_like(x)
    lut = np.ascontiguousarray(exp_lut, np.uint16)
    lib().oracle_lut_softmax_i16(_p(x), _p(out), x.shape[0], x.shape[1], _p(lut))
    return out


def requant_i16(a, mult, shift):
    a = np.ascontiguousarray(a, np.int32)
    out = np.zeros(a.shape, np.int16)
    lib().oracle_requant_i16(_p(a), _p(out), C.c_int64(a.size), C.c_int32(mult), shift)
    return out


def norm_requant_i8(a, nmult, nshift, mult, shift, zp=0):
    a = np.ascontiguousarray(a, np.int8).ravel()
    nm, ns = np.ascontiguousarray(nmult, np.int32), np.ascontiguousarray(nshift, np.int32)
    out = np.zeros_like(a)
    lib().oracle_norm_requant_i8(_p(a), _p(out), C.c_int64(a.size), nm.size, _p(nm), _p(ns),
                                 C.c_int32(mult), shift, zp)
    return out


def gemm_softmax_u8(A, B, exp_lut, b_transposed=False, requant=False, mult=1, shift=0):
    sc = (gemm_i8_rq_ex(A, B, mult, shift, 0, b_transposed=b_transposed) if requant
          else gemm_i8_acc(A, B, "i8_sat", b_transposed=b_transposed))
    return lut_softmax_u8(sc, exp_lut)


def gelu_ffn_residual_i8(x, W1, b1, gelu_lut, W2, b2, x_res, gamma, beta, inv_lut):
    hid = gemm_i8_acc(x, W1, "lut_i8", bias=b1, lut=gelu_lut)
    s = gemm_i8_acc(hid, W2, "i8_sat", bias=b2, res=np.ascontiguousarray(x_res, np.int8))
    return layernorm_lut_i8(s, gamma, beta, inv_lut)


def rmsnorm_f16(x, gamma, eps):
    x = np.ascontiguousarray(x, np.float16)
    g = np.ascontiguousarray(gamma, np.float16)
    out = np.zeros_like(x)
    R, Cc = x.shape
    lib().oracle_rmsnorm_f16_rows(_p(x), _p(g), _p(out), R, Cc, C.c_float(eps), 0, R)
    return out


def kv_cache_update_i8(k_cache, v_cache, k_new, v_new, pos):
    k_cache, v_cache = np.array(k_cache, np.int8), np.array(v_cache, np.int8)
    heads, cache_len, head_dim = k_cache.shape
    k_new, v_new = np.ascontiguousarray(k_new, np.int8), np.ascontiguousarray(v_new, np.int8)
    lib().oracle_kv_cache_update_i8(_p(k_cache), _p(v_cache), _p(k_new), _p(v_new), pos, heads,
                                    cache_len, head_dim)
    return k_cache, v_cache


def rope_pair_f16(x, cos_t, sin_t):
    x = np.ascontiguousarray(x, np.float16).ravel()
    cos_t, sin_t = np.ascontiguousarray(cos_t, np.float16), np.ascontiguousarray(sin_t, np.float16)
    out = np.zeros_like(x)
    lib().oracle_rope_pair_f16(_p(x), _p(cos_t), _p(sin_t), _p(out), C.c_int64(x.size // 2))
    return out


def ffn_hmx_i8(X, W1, b1, W2, b2, sh1=8, sh2=3):
    X = np.ascontiguousarray(X, np.uint8)
    W1, W2 = np.ascontiguousarray(W1, np.int8), np.ascontiguousarray(W2, np.int8)
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    (M, D), F = X.shape, W1.shape[1]
    out = np.zeros((M, D), np.int8)
    lib().oracle_ffn_hmx_i8(_p(X), _p(W1), _p(b1), _p(W2), _p(b2), _p(out), M, D, F, sh1, sh2)
    return out


def ffn_swiglu_hmx_i8(X, Wg, Wu, Wd, bd, silu_lut, sg=2, su=2, sh=10, zp=8, so=3):
    X = np.ascontiguousarray(X, np.uint8)
    Wg, Wu, Wd = (np.ascontiguousarray(w, np.int8) for w in (Wg, Wu, Wd))
    bd, silu_lut = np.ascontiguousarray(bd, np.int32), np.ascontiguousarray(silu_lut, np.uint8)
    (M, D), F = X.shape, Wg.shape[1]
    out = np.zeros((M, D), np.int8)
    lib().oracle_ffn_swiglu_hmx_i8(_p(X), _p(Wg), _p(Wu), _p(Wd), _p(bd), _p(silu_lut), _p(out), M,
                                   D, F, sg, su, sh, zp, so)
    return out


def encoder_block_i8(X, W1, b1, W2, b2, exp_lut):
    X = np.ascontiguousarray(X, np.uint8)
    W1, W2 = np.ascontiguousarray(W1, np.int8), np.ascontiguousarray(W2, np.int8)
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    exp_lut = np.ascontiguousarray(exp_lut, np.uint8)
    S, D = X.shape
    F = W1.shape[1]
    out = np.zeros((S, D), np.int8)
    lib().oracle_encoder_block_i8(_p(X), _p(W1), _p(b1), _p(W2), _p(b2), _p(exp_lut), _p(out), S, D, F)
    return out


def affine_ew(x, out_dtype, zp_in=0, mult=1, add=0, shift=0, round="half_away", wrap32=False,
              zp_out=0, lo=None, hi=None):
    x = np.ascontiguousarray(x)
    info = np.iinfo(out_dtype)
    lo = info.min if lo is None else lo
    hi = info.max if hi is None else hi
    out = np.zeros(x.shape, out_dtype)
    lib().oracle_affine_ew(_p(x), ELEM[x.dtype], _p(out), ELEM[np.dtype(out_dtype)],
                           C.c_int64(x.size), C.c_int32(zp_in), C.c_int32(mult), C.c_int64(add),
                           shift, {"half_away": 0, "floor": 1}[round], int(wrap32), zp_out,
                           C.c_int32(lo), C.c_int32(hi))
    return out


def gemm_i16(A, B):
    A, B = np.ascontiguousarray(A, np.int16), np.ascontiguousarray(B, np.int16)
    (M, K), N = A.shape, B.shape[1]
    C_ = np.zeros((M, N), np.int32)
    lib().oracle_gemm_i16(_p(A), _p(B), _p(C_), M, N, K)
    return C_


def mix_mlp_i8(X, W1, b1, W2, b2, mult1, shift1, mult2, shift2, lut=None):
    X, W1, W2 = (np.ascontiguousarray(a, np.int8) for a in (X, W1, W2))
    b1, b2 = np.ascontiguousarray(b1, np.int32), np.ascontiguousarray(b2, np.int32)
    (M, K), V, D = X.shape, W1.shape[0], W2.shape[0]
    out = np.zeros((M, D), np.int8)
    lp = _p(np.ascontiguousarray(lut, np.int8)) if lut is not None else None
    lib().oracle_mix_mlp_i8(_p(X), _p(W1), _p(b1), lp, _p(W2), _p(b2), _p(out), M, K, V, D,
                            C.c_int32(mult1), shift1, C.c_int32(mult2), shift2)
    return out


def token_mix_i8(X, W, b, W2, b2, mult1, shift1, mult2, shift2):
    X, W, W2 = (np.ascontiguousarray(a, np.int8) for a in (X, W, W2))
    b, b2 = np.ascontiguousarray(b, np.int32), np.ascontiguousarray(b2, np.int32)
    (T, Cc), DM = X.shape, W.shape[0]
    out = np.zeros((T, Cc), np.int8)
    lib().oracle_token_mix_i8(_p(X), _p(W), _p(b), _p(W2), _p(b2), _p(out), T, Cc, DM,
                              C.c_int32(mult1), shift1, C.c_int32(mult2), shift2)
    return out


def rnn_cell_i8(Wx, Wh, b, x, h_prev, mult, shift, zp, tanh_lut):
    Wx, Wh, x, h_prev, tanh_lut = (np.ascontiguousarray(a, np.int8) for a in (Wx, Wh, x, h_prev, tanh_lut))
    b = np.ascontiguousarray(b, np.int32)
    H, I = Wx.shape
    out = np.zeros(H, np.int8)
    lib().oracle_rnn_cell_i8(_p(Wx), _p(Wh), _p(b), _p(x), _p(h_prev), _p(out), H, I,
                             C.c_int32(mult), shift, zp, _p(tanh_lut))
    return out


def conv2d_hmx(x, W, bias=None, store="u16_field", act="none", stride=1):
    x, W = np.ascontiguousarray(x, np.uint8), np.ascontiguousarray(W, np.int8)
    c_in, ih, iw = x.shape
    c_out, _, kh, kw = W.shape
    kind, dt = HMX_STORE[store]
    oh, ow = (ih - kh) // stride + 1, (iw - kw) // stride + 1
    out = np.zeros((c_out, oh, ow), dt)
    bp = _p(np.ascontiguousarray(bias, np.int32)) if bias is not None else None
    lib().oracle_conv2d_hmx(_p(x), _p(W), bp, _p(out), kind, HMX_ACT[act], c_in, ih, iw, c_out, kh, kw,
                            stride)
    return out
