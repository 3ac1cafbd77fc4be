"""NumPy-level operators over libhexcuda's host-pointer entries.

Each function mirrors one corpus task's ``candidate_kernel`` (same argument
meaning, same result) and runs it on the initialised B200 devices, rows
sharded across them.  fp16 data is ``numpy.float16``.  Errors raise
``HexcudaError``; nothing falls back to the CPU.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, load


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype != np.dtype(dtype):
        raise TypeError(f"expected {np.dtype(dtype)}, got {a.dtype}")
    return a


def init(ngpus: int = 0) -> int:
    """Initialise devices 0..ngpus-1 (0 = all); returns the device count."""
    lib = load()
    check(lib.hexcuda_init(ngpus))
    return lib.hexcuda_device_count()


def init_devices(devs) -> int:
    lib = load()
    arr = (C.c_int * len(devs))(*devs)
    check(lib.hexcuda_init_devices(arr, len(devs)))
    return lib.hexcuda_device_count()


def last_kernel_ms() -> float:
    return float(load().hexcuda_last_kernel_ms())


# ------------------------------------------------- shards and replicated outputs

def shard_rows(rows: int, nparts: int, part: int) -> tuple[int, int]:
    """Rows [r0, r1) of part `part` of `nparts` (the split every entry uses)."""
    r0, r1 = C.c_int64(), C.c_int64()
    check(load().hexcuda_shard_rows(rows, nparts, part, C.byref(r0), C.byref(r1)))
    return r0.value, r1.value


def set_replicate(on: bool) -> None:
    """Ask the host entries to also all-gather their (row-major) outputs over
    NVLink, so that every initialised device holds the whole output."""
    check(load().hexcuda_set_replicate(int(bool(on))))


def replica(dev: int, shape, dtype) -> np.ndarray:
    """Copy device slot `dev`'s replica of the last host entry's output."""
    lib = load()
    ptr, nbytes = C.c_void_p(), C.c_size_t()
    check(lib.hexcuda_replica(dev, C.byref(ptr), C.byref(nbytes)))
    out = np.empty(shape, dtype)
    if out.nbytes != nbytes.value:
        raise ValueError(f"replica holds {nbytes.value} bytes, {out.nbytes} requested")
    check(lib.hexcuda_d2h(dev, _p(out), ptr, out.nbytes))
    check(lib.hexcuda_sync(dev))
    return out


def last_collective_ms() -> float:
    return float(load().hexcuda_last_collective_ms())


# ----------------------------------------------------------- integer family

def gemm_i8_requant(A, B, mult: int, shift: int, zp: int) -> np.ndarray:
    """i8_gemm_requant: A [M,K] s8, B [K,N] s8 -> [M,N] s8."""
    A, B = _c(A, np.int8), _c(B, np.int8)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2
    out = np.empty((M, N), np.int8)
    check(load().hexcuda_host_gemm_i8_requant(_p(A), _p(B), _p(out), M, N, K, mult, shift, zp))
    return out


def gemm_i8_bias_requant(A, B, bias, mult: int, shift: int, zp: int) -> np.ndarray:
    A, B, bias = _c(A, np.int8), _c(B, np.int8), _c(bias, np.int32)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2 and bias.shape == (N,)
    out = np.empty((M, N), np.int8)
    check(load().hexcuda_host_gemm_i8_bias_requant(_p(A), _p(B), _p(bias), _p(out), M, N, K, mult,
                                                   shift, zp))
    return out


def gemm_i8_zp(A, B, zpA: int, scale_mult: int, scale_shift: int) -> np.ndarray:
    A, B = _c(A, np.int8), _c(B, np.int8)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2
    out = np.empty((M, N), np.int8)
    check(load().hexcuda_host_gemm_i8_zp(_p(A), _p(B), _p(out), M, N, K, zpA, scale_mult,
                                         scale_shift))
    return out


def gemm_u8s8_pc(A, B, bias, zpA: int, mult, shift, zp_out: int) -> np.ndarray:
    A, B = _c(A, np.uint8), _c(B, np.int8)
    bias, mult, shift = _c(bias, np.int32), _c(mult, np.int32), _c(shift, np.int32)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2 and bias.shape == mult.shape == shift.shape == (N,)
    out = np.empty((M, N), np.uint8)
    check(load().hexcuda_host_gemm_u8s8_pc(_p(A), _p(B), _p(bias), _p(out), M, N, K, zpA,
                                           _p(mult), _p(shift), zp_out))
    return out


HMX_OUT_I32, HMX_OUT_I8, HMX_OUT_U8_BIAS_RELU = 0, 1, 2


def gemm_hmx(A, B, out_kind: int = HMX_OUT_I32, bias=None, zpA: int = 0,
             b_transposed: bool = False) -> np.ndarray:
    """HMX-convention u8 x s8 GEMM: sx12((acc * 17 + 8) >> 4) of
    acc = (A - zpA) . B, then int32 / int8-clamp / u8 bias-ReLU by out_kind.
    B is [K, N], or Bt [N, K] when b_transposed."""
    A, B = _c(A, np.uint8), _c(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    assert (B.shape[1] if b_transposed else B.shape[0]) == K
    dt = {HMX_OUT_I32: np.int32, HMX_OUT_I8: np.int8, HMX_OUT_U8_BIAS_RELU: np.uint8}[out_kind]
    out = np.empty((M, N), dt)
    if out_kind == HMX_OUT_U8_BIAS_RELU:
        bias = _c(bias, np.int32)
        assert bias.shape == (N,)
    check(load().hexcuda_host_gemm_hmx(_p(A), _p(B), int(b_transposed),
                                       _p(bias) if bias is not None else None, _p(out), out_kind,
                                       M, N, K, zpA))
    return out


HMX_STORE = {"i32": (0, np.int32), "i8_sat": (1, np.int8), "u8_sat": (2, np.uint8),
             "i8_low": (3, np.int8), "u16_field": (4, np.uint16), "lut_i32": (5, np.int32),
             "lut_i8": (6, np.int8), "acc_i32": (7, np.int32)}
HMX_ACT = {"none": 0, "relu": 1, "leaky_shr3": 2}


def gemm_hmx_ex(A, B, store: str = "i32", act: str = "none", bias=None, res=None, lut=None,
                zpA: int = 0, b_transposed: bool = False, col_major: bool = False) -> np.ndarray:
    """HMX-convention u8 x s8 GEMM with the family's post-ops: sx12 field,
    + bias[j], + res[i][j] (int32 or int8 [M, N]), activation, store kind
    (keys of HMX_STORE).  Returns [M, N], or its transpose's memory [N, M]
    when col_major."""
    A, B = _c(A, np.uint8), _c(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    kind, dt = HMX_STORE[store]
    out = np.empty((N, M) if col_major else (M, N), dt)
    res_kind = 0
    if res is not None:
        res = np.ascontiguousarray(res)
        res_kind = {np.dtype(np.int32): 1, np.dtype(np.int8): 2}[res.dtype]
        assert res.shape == (M, N)
    if bias is not None:
        bias = _c(bias, np.int32)
    if lut is not None:
        lut = _c(lut, np.int32 if store == "lut_i32" else np.int8)
        assert lut.shape == (256,)
    pp = lambda a: _p(a) if a is not None else None
    check(load().hexcuda_host_gemm_hmx_ex(_p(A), _p(B), int(b_transposed), pp(bias), pp(res),
                                          res_kind, pp(lut), _p(out), kind, HMX_ACT[act],
                                          int(col_major), M, N, K, zpA))
    return out


RQ_PRE = {"a": 0, "add": 1, "add_relu": 2, "mul_add": 3}


def requant_ew(a, b=None, pre: str = "a", pre_c: int = 0, mult: int = 1, shift: int = 0,
               zp: int = 0, sign_of_a: bool = False, lo1: int = -128, hi1: int = 127,
               lo2: int = -128, hi2: int = 127, lut=None, out_dtype=np.int8) -> np.ndarray:
    """Elementwise requant family: pre-op of a (and b), round-half-away
    requant, two clamps, optional 256-entry int8 table; one byte out."""
    a = np.ascontiguousarray(a)
    assert a.dtype in (np.int32, np.int8)
    b_kind = 0
    if b is not None:
        b = np.ascontiguousarray(b)
        assert b.shape == a.shape
        b_kind = {np.dtype(np.int32): 1, np.dtype(np.int8): 2}[b.dtype]
    if lut is not None:
        lut = _c(lut, np.int8)
        assert lut.shape == (256,)
    out = np.empty(a.shape, out_dtype)
    check(load().hexcuda_host_requant_ew(_p(a), int(a.dtype == np.int8),
                                         _p(b) if b is not None else None, b_kind, _p(out), a.size,
                                         RQ_PRE[pre], pre_c, mult, shift, zp, int(sign_of_a), lo1,
                                         hi1, lo2, hi2, _p(lut) if lut is not None else None))
    return out


def epilogue_bias_i32(acc, bias) -> np.ndarray:
    acc, bias = _c(acc, np.int32), _c(bias, np.int32)
    R, Cc = acc.shape
    out = np.empty_like(acc)
    check(load().hexcuda_host_epilogue_bias_i32(_p(acc), _p(bias), _p(out), R, Cc))
    return out


def relu_i8(x) -> np.ndarray:
    x = _c(x, np.int8)
    out = np.empty_like(x)
    check(load().hexcuda_host_relu_i8(_p(x), _p(out), x.size))
    return out


ELEM = {np.dtype(np.int8): 0, np.dtype(np.uint8): 1, np.dtype(np.int16): 2,
        np.dtype(np.int32): 3}
RED_OPS = {"sum": 0, "sum64": 1, "sumsq": 2, "sumsq_diff": 3, "dot": 4, "l1": 5, "absmax": 6,
           "max": 7, "min": 8, "argmax": 9, "argmin": 10, "top1": 11, "mean": 12}


def reduce_int(a, op: str, b=None):
    """Whole-array integer reduction (hexcuda_host_reduce_int) of an int8,
    uint8, int16 or int32 array; returns an int, or (max, first index) for
    "top1"."""
    a = np.ascontiguousarray(a).ravel()
    if b is not None:
        b = _c(b, a.dtype).ravel()
        assert b.size == a.size
    out = np.zeros(2, np.int64 if op == "sum64" else np.int32)
    check(load().hexcuda_host_reduce_int(_p(a), None if b is None else _p(b), ELEM[a.dtype],
                                         a.size, RED_OPS[op], _p(out)))
    return (int(out[0]), int(out[1])) if op == "top1" else int(out[0])


def minmax_ew(a, b=None, c: int = 0, op: str = "max") -> np.ndarray:
    """Elementwise max / min of a and b, or of a and the scalar c (b None)."""
    a = np.ascontiguousarray(a)
    if b is not None:
        b = _c(b, a.dtype)
        assert b.shape == a.shape
    out = np.empty_like(a)
    check(load().hexcuda_host_minmax_ew(_p(a), None if b is None else _p(b), int(c), ELEM[a.dtype],
                                        {"max": 0, "min": 1}[op], _p(out), a.size))
    return out


def group_sum_i8(a, w: int = 4) -> np.ndarray:
    """out[k] = sum of a[w k : w k + w] (int8 -> int32)."""
    a = _c(a, np.int8).ravel()
    g = a.size // w
    out = np.empty(g, np.int32)
    check(load().hexcuda_host_group_sum_i8(_p(a), _p(out), g, w))
    return out


def group_dot_i8(a, b, w: int = 4) -> np.ndarray:
    """out[k] = sum_j a[w k + j] b[w k + j] (int8 x int8 -> int32)."""
    a = _c(a, np.int8).ravel()
    b = _c(b, np.int8).ravel()
    assert a.size == b.size
    g = a.size // w
    out = np.empty(g, np.int32)
    check(load().hexcuda_host_group_dot_i8(_p(a), _p(b), _p(out), g, w))
    return out


def gate_mul_requant_i8(gate, up, lut, mult: int, shift: int) -> np.ndarray:
    """SiLU-gated product: sat8(round_half_away(lut[gate + 128] up * mult >> shift))."""
    gate, up, lut = _c(gate, np.int8), _c(up, np.int8), _c(lut, np.int8)
    assert gate.shape == up.shape and lut.shape == (256,)
    out = np.empty(gate.shape, np.int8)
    check(load().hexcuda_host_gate_mul_requant_i8(_p(gate), _p(up), _p(lut), _p(out), gate.size,
                                                  mult, shift))
    return out


def scan_max_i8(x) -> np.ndarray:
    """Inclusive prefix maximum of an int8 array."""
    x = _c(x, np.int8).ravel()
    out = np.empty_like(x)
    check(load().hexcuda_host_scan_max_i8(_p(x), _p(out), x.size))
    return out


def head_group_reduce_i8(X, G: int, mult: int, shift: int) -> np.ndarray:
    """Y[g] = sat_i8(round_half_away(sum of the H/G head planes of group g
    * mult >> shift)); X [H, ...] int8 -> Y [G, ...]."""
    X = _c(X, np.int8)
    H = X.shape[0]
    MN = int(np.prod(X.shape[1:]))
    Y = np.empty((G,) + X.shape[1:], np.int8)
    check(load().hexcuda_host_head_group_reduce_i8(_p(X), _p(Y), H, G, MN, int(mult), shift))
    return Y


LN_AFFINE = {"shared": 0, "rowwise": 1, "per_row": 2, "rms": 3}


def layernorm_lut_i8(x, gamma, beta, inv_lut, affine: str = "shared", res=None, idx=None):
    """int8 layernorm with an inverse-variance table (hexcuda_layernorm_lut_i8)
    over the rows of x [R, W]; with idx, the rows x[idx[r]] (x is the table)."""
    x = _c(x, np.int8)
    xrows, W = x.shape
    idx = _c(idx, np.int32) if idx is not None else None
    R = idx.size if idx is not None else xrows
    res = _c(res, np.int8) if res is not None else None
    gamma, inv_lut = _c(gamma, np.int8), _c(inv_lut, np.uint8)
    beta = _c(beta, np.int8) if beta is not None else None
    out = np.empty((R, W), np.int8)
    check(load().hexcuda_host_layernorm_lut_i8(_p(x), xrows, None if idx is None else _p(idx),
                                               None if res is None else _p(res), _p(out), R, W,
                                               _p(gamma), None if beta is None else _p(beta),
                                               _p(inv_lut), LN_AFFINE[affine]))
    return out


def layernorm_lut_i16(x, gamma, beta, inv_lut, order: int = 0) -> np.ndarray:
    x = _c(x, np.int16)
    R, Cc = x.shape
    out = np.empty_like(x)
    check(load().hexcuda_host_layernorm_lut_i16(_p(x), _p(out), R, Cc, _p(_c(gamma, np.int16)),
                                                _p(_c(beta, np.int16)), _p(_c(inv_lut, np.uint16)),
                                                order))
    return out


def lut_softmax_u8(x, exp_lut, recip_lut=None) -> np.ndarray:
    x = _c(x, np.int8)
    R, Cc = x.shape
    out = np.empty((R, Cc), np.uint8)
    rl = _c(recip_lut, np.uint16) if recip_lut is not None else None
    check(load().hexcuda_host_lut_softmax_u8(_p(x), _p(out), R, Cc, _p(_c(exp_lut, np.uint8)),
                                             None if rl is None else _p(rl)))
    return out


def lut_softmax_i16(x, exp_lut) -> np.ndarray:
    x = _c(x, np.int16)
    R, Cc = x.shape
    out = np.empty_like(x)
    check(load().hexcuda_host_lut_softmax_i16(_p(x), _p(out), R, Cc, _p(_c(exp_lut, np.uint16))))
    return out


def requant_i16(a, mult: int, shift: int) -> np.ndarray:
    a = _c(a, np.int32)
    out = np.empty(a.shape, np.int16)
    check(load().hexcuda_host_requant_i16(_p(a), _p(out), a.size, mult, shift))
    return out


def norm_requant_i8(a, nmult, nshift, mult: int, shift: int, zp: int = 0) -> np.ndarray:
    """Per-channel requant (channels = equal parts of a) then a second one;
    elements past the channels' last whole part are returned as zero."""
    a = _c(a, np.int8).ravel()
    nmult, nshift = _c(nmult, np.int32), _c(nshift, np.int32)
    out = np.zeros_like(a)
    check(load().hexcuda_host_norm_requant_i8(_p(a), _p(out), a.size, nmult.size, _p(nmult),
                                              _p(nshift), mult, shift, zp))
    return out


def gemm_softmax_u8(A, B, exp_lut, b_transposed: bool = False, requant: bool = False,
                    mult: int = 1, shift: int = 0) -> np.ndarray:
    A, B = _c(A, np.int8), _c(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    out = np.empty((M, N), np.uint8)
    check(load().hexcuda_host_gemm_softmax_u8(_p(A), _p(B), int(b_transposed),
                                              _p(_c(exp_lut, np.uint8)), _p(out), M, N, K,
                                              int(requant), mult, shift))
    return out


def gelu_ffn_residual_i8(x, W1, b1, gelu_lut, W2, b2, x_res, gamma, beta, inv_lut) -> np.ndarray:
    x, W1, W2, x_res = (_c(t, np.int8) for t in (x, W1, W2, x_res))
    (M, K), (_, V), (_, D) = x.shape, W1.shape, W2.shape
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_gelu_ffn_residual_i8(
        _p(x), _p(W1), _p(_c(b1, np.int32)), _p(_c(gelu_lut, np.int8)), _p(W2),
        _p(_c(b2, np.int32)), _p(x_res), _p(_c(gamma, np.int8)), _p(_c(beta, np.int8)),
        _p(_c(inv_lut, np.uint8)), _p(out), M, K, V, D))
    return out


def attn_qkt_av_hmx(Q, K, V) -> np.ndarray:
    """sx12 field of (sx12 field of Q K^T) V; Q [SQ, D] u8, K / V [SK, D] s8."""
    Q, K, V = _c(Q, np.uint8), _c(K, np.int8), _c(V, np.int8)
    (SQ, D), (SK, D2) = Q.shape, K.shape
    assert D == D2 and V.shape == K.shape
    out = np.empty((SQ, D), np.int32)
    check(load().hexcuda_host_attn_qkt_av_hmx(_p(Q), _p(K), _p(V), _p(out), SQ, SK, D))
    return out


ATTN_LUT = {"requant": 0, "hmx": 1, "hmx_rope": 2}


def attn_lut_i8(mode: str, Q, K, V, exp_lut, cos_lut=None, sin_lut=None, rot_shift: int = 0,
                scale_mult: int = 0, scale_shift: int = 0, av_mult: int = 0,
                av_shift: int = 0) -> np.ndarray:
    """int8 attention with the exp-table softmax; Q [HQ, S, D] (int8 for
    "requant", u8 otherwise), K / V [HKV, S, D] int8."""
    m = ATTN_LUT[mode]
    Q = _c(Q, np.int8 if m == 0 else np.uint8)
    K, V = _c(K, np.int8), _c(V, np.int8)
    exp_lut = _c(exp_lut, np.uint8)
    HQ, S, D = Q.shape
    out = np.empty(Q.shape, np.int8 if m == 0 else np.uint16)
    cs = _c(cos_lut, np.int8) if cos_lut is not None else None
    sn = _c(sin_lut, np.int8) if sin_lut is not None else None
    check(load().hexcuda_host_attn_lut_i8(m, _p(Q), _p(K), _p(V), _p(exp_lut),
                                          _p(cs) if cs is not None else None,
                                          _p(sn) if sn is not None else None, rot_shift, _p(out),
                                          HQ, K.shape[0], S, D, scale_mult, scale_shift, av_mult,
                                          av_shift))
    return out


def attn_lut_i8_window(Q, K, V, exp_lut, window: int, scale_mult: int, scale_shift: int,
                       av_mult: int, av_shift: int) -> np.ndarray:
    """int8 LUT-softmax attention (requant scores and output) with a banded
    mask: scores of keys with |i - j| > window are -128.  Q / K / V [H, S, D]."""
    Q, K, V = _c(Q, np.int8), _c(K, np.int8), _c(V, np.int8)
    assert Q.shape == K.shape == V.shape and Q.ndim == 3
    H, S, D = Q.shape
    out = np.empty(Q.shape, np.int8)
    check(load().hexcuda_host_attn_lut_i8_window(_p(Q), _p(K), _p(V), _p(_c(exp_lut, np.uint8)),
                                                 _p(out), H, S, D, window, scale_mult, scale_shift,
                                                 av_mult, av_shift))
    return out


ROUND = {"half_away": 0, "floor": 1}


def affine_ew(x, out_dtype, zp_in: int = 0, mult: int = 1, add: int = 0, shift: int = 0,
              round: str = "half_away", wrap32: bool = False, zp_out: int = 0, lo=None,
              hi=None) -> np.ndarray:
    """clamp(round((x - zp_in) * mult + add, shift) + zp_out, lo, hi) in the
    integer type out_dtype (lo / hi default to its range)."""
    x = np.ascontiguousarray(x)
    info = np.iinfo(out_dtype)
    lo = info.min if lo is None else lo
    hi = info.max if hi is None else hi
    out = np.empty(x.shape, out_dtype)
    check(load().hexcuda_host_affine_ew(_p(x), ELEM[x.dtype], _p(out), ELEM[np.dtype(out_dtype)],
                                        x.size, zp_in, mult, add, shift, ROUND[round], int(wrap32),
                                        zp_out, lo, hi))
    return out


def kv_cache_update_i8(k_cache, v_cache, k_new, v_new, pos: int):
    """Writes k_new / v_new [heads, head_dim] into row pos of the caches
    [heads, cache_len, head_dim] (in place on the host arrays, which are
    returned)."""
    assert k_cache.dtype == v_cache.dtype == np.int8 and k_cache.flags.c_contiguous
    assert v_cache.flags.c_contiguous and k_cache.shape == v_cache.shape
    heads, cache_len, head_dim = k_cache.shape
    k_new, v_new = _c(k_new, np.int8), _c(v_new, np.int8)
    assert k_new.shape == v_new.shape == (heads, head_dim)
    check(load().hexcuda_host_kv_cache_update_i8(_p(k_cache), _p(v_cache), _p(k_new), _p(v_new), pos,
                                                 heads, cache_len, head_dim))
    return k_cache, v_cache


def rope_pair_f16(x, cos_t, sin_t) -> np.ndarray:
    """Rotary embedding of interleaved fp16 pairs (x [2 n], cos / sin [n])."""
    x, cos_t, sin_t = _c(x, np.float16).ravel(), _c(cos_t, np.float16), _c(sin_t, np.float16)
    n = x.size // 2
    assert x.size == 2 * n and cos_t.size == sin_t.size == n
    out = np.empty_like(x)
    check(load().hexcuda_host_rope_pair_f16(_p(x), _p(cos_t), _p(sin_t), _p(out), n))
    return out


def conv2d_hmx(x, W, bias=None, store: str = "u16_field", act: str = "none", stride: int = 1):
    """HMX-convention convolution, no padding: x [c_in, ih, iw] u8, W
    [c_out, c_in, kh, kw] int8 -> [c_out, oh, ow] (store "u16_field",
    "i32" or "i8_sat"; activation as gemm_hmx_ex)."""
    x, W = _c(x, np.uint8), _c(W, np.int8)
    c_in, ih, iw = x.shape
    c_out, c_in2, kh, kw = W.shape
    assert c_in == c_in2
    kind, dt = HMX_STORE[store]
    oh, ow = (ih - kh) // stride + 1, (iw - kw) // stride + 1
    bp = _p(_c(bias, np.int32)) if bias is not None else None
    out = np.empty((c_out, oh, ow), dt)
    check(load().hexcuda_host_conv2d_hmx(_p(x), _p(W), bp, _p(out), kind, HMX_ACT[act], c_in, ih, iw,
                                         c_out, kh, kw, stride))
    return out


def gemm_i16(A, B) -> np.ndarray:
    """int16 GEMM, int32 accumulator (modulo 2^32): A [M, K], B [K, N]."""
    A, B = _c(A, np.int16), _c(B, np.int16)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2
    C = np.empty((M, N), np.int32)
    check(load().hexcuda_host_gemm_i16(_p(A), _p(B), _p(C), M, N, K))
    return C


def mix_mlp_i8(X, W1, b1, W2, b2, mult1: int, shift1: int, mult2: int, shift2: int,
               lut=None) -> np.ndarray:
    """Channel-mixing MLP: two requantised products with Bt weights (W1
    [V, K], W2 [D, V]) and an optional int8 table between them."""
    X, W1, W2 = _c(X, np.int8), _c(W1, np.int8), _c(W2, np.int8)
    b1, b2 = _c(b1, np.int32), _c(b2, np.int32)
    (M, K), (V, K2), (D, V2) = X.shape, W1.shape, W2.shape
    assert K == K2 and V == V2
    lp = _p(_c(lut, np.int8)) if lut is not None else None
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_mix_mlp_i8(_p(X), _p(W1), _p(b1), lp, _p(W2), _p(b2), _p(out), M, K, V,
                                         D, mult1, shift1, mult2, shift2))
    return out


def token_mix_i8(X, W, b, W2, b2, mult1: int, shift1: int, mult2: int, shift2: int) -> np.ndarray:
    """Token-mixing MLP of X [T, C]: W [DM, T], W2 [T, DM]."""
    X, W, W2 = _c(X, np.int8), _c(W, np.int8), _c(W2, np.int8)
    b, b2 = _c(b, np.int32), _c(b2, np.int32)
    (T, Cc), DM = X.shape, W.shape[0]
    out = np.empty((T, Cc), np.int8)
    check(load().hexcuda_host_token_mix_i8(_p(X), _p(W), _p(b), _p(W2), _p(b2), _p(out), T, Cc, DM,
                                           mult1, shift1, mult2, shift2))
    return out


def rnn_cell_i8(Wx, Wh, b, x, h_prev, mult: int, shift: int, zp: int, tanh_lut) -> np.ndarray:
    """One int8 RNN step: tanh table of the requantised b + Wx x + Wh h."""
    Wx, Wh, x, h_prev = _c(Wx, np.int8), _c(Wh, np.int8), _c(x, np.int8), _c(h_prev, np.int8)
    b, tanh_lut = _c(b, np.int32), _c(tanh_lut, np.int8)
    H, I = Wx.shape
    out = np.empty(H, np.int8)
    check(load().hexcuda_host_rnn_cell_i8(_p(Wx), _p(Wh), _p(b), _p(x), _p(h_prev), _p(out), H, I,
                                          mult, shift, zp, _p(tanh_lut)))
    return out


def ffn_hmx_i8(X, W1, b1, W2, b2, sh1: int = 8, sh2: int = 3) -> np.ndarray:
    """HMX-convention two-layer FFN (ReLU + shift between, shift + saturate
    after); X u8 [M, D], W1 [D, Dff], W2 [Dff, D]."""
    X, W1, W2 = _c(X, np.uint8), _c(W1, np.int8), _c(W2, np.int8)
    b1, b2 = _c(b1, np.int32), _c(b2, np.int32)
    (M, D), (D2, F), (F2, D3) = X.shape, W1.shape, W2.shape
    assert D == D2 == D3 and F == F2 and b1.size == F and b2.size == D
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_ffn_hmx_i8(_p(X), _p(W1), _p(b1), _p(W2), _p(b2), _p(out), M, D, F,
                                         sh1, sh2))
    return out


def ffn_swiglu_hmx_i8(X, Wg, Wu, Wd, bd, silu_lut, sg: int = 2, su: int = 2, sh: int = 10,
                      zp: int = 8, so: int = 3) -> np.ndarray:
    """HMX-convention SwiGLU FFN (gate / up projections, SiLU-table gate x up
    with a zero point, down projection + bias + shift + saturate)."""
    X, Wg, Wu, Wd = _c(X, np.uint8), _c(Wg, np.int8), _c(Wu, np.int8), _c(Wd, np.int8)
    bd, silu_lut = _c(bd, np.int32), _c(silu_lut, np.uint8)
    (M, D), (D2, F) = X.shape, Wg.shape
    assert D == D2 and Wu.shape == Wg.shape and Wd.shape == (F, D) and bd.size == D
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_ffn_swiglu_hmx_i8(_p(X), _p(Wg), _p(Wu), _p(Wd), _p(bd), _p(silu_lut),
                                                _p(out), M, D, F, sg, su, sh, zp, so))
    return out


def encoder_block_i8(X, W1, b1, W2, b2, exp_lut) -> np.ndarray:
    """int8 encoder block: HMX-field self-attention of X with itself over
    every key, residual, HMX-field FFN, residual."""
    X, W1, W2 = _c(X, np.uint8), _c(W1, np.int8), _c(W2, np.int8)
    b1, b2, exp_lut = _c(b1, np.int32), _c(b2, np.int32), _c(exp_lut, np.uint8)
    S, D = X.shape
    F = W1.shape[1]
    out = np.empty((S, D), np.int8)
    check(load().hexcuda_host_encoder_block_i8(_p(X), _p(W1), _p(b1), _p(W2), _p(b2), _p(exp_lut),
                                               _p(out), S, D, F))
    return out


def decoder_block_i8(X, W1, b1, act_lut, W2, b2, exp_lut) -> np.ndarray:
    X, W1, W2 = _c(X, np.uint8), _c(W1, np.int8), _c(W2, np.int8)
    b1, b2 = _c(b1, np.int32), _c(b2, np.int32)
    act_lut, exp_lut = _c(act_lut, np.int8), _c(exp_lut, np.uint8)
    S, D = X.shape
    out = np.empty((S, D), np.int8)
    check(load().hexcuda_host_decoder_block_i8(_p(X), _p(W1), _p(b1), _p(act_lut), _p(W2), _p(b2),
                                               _p(exp_lut), _p(out), S, D, W1.shape[1]))
    return out


F16_ACT = {"none": 0, "relu": 1, "leaky": 2, "gelu": 3, "sigmoid": 4, "tanh": 5}
F16_PREROUND = {False: 0, True: 1, "sum": 1, "acc": 2}


def gemm_f16_ex(A, B, act: str = "none", preround: bool = False, scale: float = 1.0, bias=None,
                res=None, b_transposed: bool = False) -> np.ndarray:
    """fp16 GEMM with the corpus's fp16 post-ops (residual, bias, rounding,
    activation, scale); B [K, N] or Bt [N, K]."""
    A, B = _c(A, np.float16), _c(B, np.float16)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    bias = _c(bias, np.float16) if bias is not None else None
    res = _c(res, np.float16) if res is not None else None
    out = np.empty((M, N), np.float16)
    check(load().hexcuda_host_gemm_f16_ex(_p(A), _p(B), int(b_transposed),
                                          _p(bias) if bias is not None else None,
                                          _p(res) if res is not None else None, _p(out),
                                          F16_ACT[act], F16_PREROUND[preround], float(scale), M, N, K))
    return out


def gemm_i8_rq_ex(A, B, mult: int, shift: int, zp: int, bias=None, relu: bool = False,
                  b_transposed: bool = False, res=None) -> np.ndarray:
    """s8 x s8 GEMM + requant, optional bias and ReLU before the requant, and
    an optional int8 residual [M, N] added with saturation after it."""
    A, B = _c(A, np.int8), _c(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    bias = _c(bias, np.int32) if bias is not None else None
    res = _c(res, np.int8) if res is not None else None
    out = np.empty((M, N), np.int8)
    check(load().hexcuda_host_gemm_i8_rq_ex(_p(A), _p(B), int(b_transposed),
                                            _p(bias) if bias is not None else None,
                                            _p(res) if res is not None else None, _p(out), M, N,
                                            K, mult, shift, zp, int(relu)))
    return out


def gemm_i8_acc(A, B, store: str = "i32", act: str = "none", bias=None, res=None, lut=None,
                b_transposed: bool = False) -> np.ndarray:
    """s8 (or u8) x s8 GEMM on the raw int32 accumulator with int64 post-ops:
    + bias[j] + res[i][j], activation, store (keys of HMX_STORE)."""
    A = np.ascontiguousarray(A)
    a_signed = {np.dtype(np.int8): 1, np.dtype(np.uint8): 0}[A.dtype]
    B = _c(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if b_transposed else B.shape[1]
    kind, dt = HMX_STORE[store]
    out = np.empty((M, N), dt)
    res_kind = 0
    if res is not None:
        res = np.ascontiguousarray(res)
        res_kind = {np.dtype(np.int32): 1, np.dtype(np.int8): 2}[res.dtype]
    if bias is not None:
        bias = _c(bias, np.int32)
    if lut is not None:
        lut = _c(lut, np.int32 if store == "lut_i32" else np.int8)
    pp = lambda a: _p(a) if a is not None else None
    check(load().hexcuda_host_gemm_i8_acc(_p(A), a_signed, _p(B), int(b_transposed), pp(bias),
                                          pp(res), res_kind, pp(lut), _p(out), kind, HMX_ACT[act],
                                          M, N, K))
    return out


def ffn_relu_i8(A, W1, b1, W2, b2, mult: int, shift: int, zp: int) -> np.ndarray:
    """Two-layer int8 FFN (GEMM + b1 + ReLU + sat8, GEMM + b2 + requant)."""
    A, W1, W2 = _c(A, np.int8), _c(W1, np.int8), _c(W2, np.int8)
    b1, b2 = _c(b1, np.int32), _c(b2, np.int32)
    (M, K), (K2, V), (V2, D) = A.shape, W1.shape, W2.shape
    assert K == K2 and V == V2
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_ffn_relu_i8(_p(A), _p(W1), _p(b1), _p(W2), _p(b2), _p(out), M, K,
                                          V, D, mult, shift, zp))
    return out


def ffn_lut_i8(A, W1, b1, act_lut, W2, b2, mult: int, shift: int, zp: int) -> np.ndarray:
    """Two-layer int8 FFN with a table activation (GEMM + b1 + sat8 + table,
    GEMM + b2 + requant)."""
    A, W1, W2, act_lut = _c(A, np.int8), _c(W1, np.int8), _c(W2, np.int8), _c(act_lut, np.int8)
    b1, b2 = _c(b1, np.int32), _c(b2, np.int32)
    (M, K), (K2, V), (V2, D) = A.shape, W1.shape, W2.shape
    assert K == K2 and V == V2 and act_lut.shape == (256,)
    out = np.empty((M, D), np.int8)
    check(load().hexcuda_host_ffn_lut_i8(_p(A), _p(W1), _p(b1), _p(act_lut), _p(W2), _p(b2), _p(out),
                                         M, K, V, D, mult, shift, zp))
    return out


def gemm_hmx_s8u8(A, B, store: str = "i32") -> np.ndarray:
    """HMX-field GEMM with s8 A [M, K] and u8 B [K, N]."""
    A, B = _c(A, np.int8), _c(B, np.uint8)
    kind, dt = {"i32": (0, np.int32), "u16_field": (4, np.uint16), "acc_i32": (7, np.int32)}[store]
    M, K = A.shape
    out = np.empty((M, B.shape[1]), dt)
    check(load().hexcuda_host_gemm_hmx_s8u8(_p(A), _p(B), _p(out), kind, M, B.shape[1], K))
    return out


def requant_per_channel(a, mult, shift, zp: int) -> np.ndarray:
    a, mult, shift = _c(a, np.int32), _c(mult, np.int32), _c(shift, np.int32)
    R, Cc = a.shape
    out = np.empty((R, Cc), np.int8)
    check(load().hexcuda_host_requant_per_channel(_p(a), _p(out), R, Cc, _p(mult), _p(shift), zp))
    return out


def requantize_i32_u8(a, mult: int, shift: int, zp: int) -> np.ndarray:
    a = _c(a, np.int32)
    out = np.empty(a.shape, np.uint8)
    check(load().hexcuda_host_requantize_i32_u8(_p(a), _p(out), a.size, mult, shift, zp))
    return out


# --------------------------------------------------------------- fp16 GEMM

def gemm_f16_nt(A, Bt) -> np.ndarray:
    """out[M,N] = A[M,K] . Bt[N,K]^T, fp32 accumulate, fp16 out."""
    A, Bt = _c(A, np.float16), _c(Bt, np.float16)
    (M, K), (N, K2) = A.shape, Bt.shape
    assert K == K2
    out = np.empty((M, N), np.float16)
    check(load().hexcuda_host_gemm_f16_nt(_p(A), _p(Bt), _p(out), M, N, K))
    return out


def gemm_f16_nn(A, B) -> np.ndarray:
    A, B = _c(A, np.float16), _c(B, np.float16)
    (M, K), (K2, N) = A.shape, B.shape
    assert K == K2
    out = np.empty((M, N), np.float16)
    check(load().hexcuda_host_gemm_f16_nn(_p(A), _p(B), _p(out), M, N, K))
    return out


# --------------------------------------------------------------- attention

def attn_f16(Q, K, V, scale: float, causal: bool) -> np.ndarray:
    """Q [..., SQ, D], K/V [..., SK, D] (leading dims flattened into heads)."""
    Q, K, V = _c(Q, np.float16), _c(K, np.float16), _c(V, np.float16)
    SQ, D = Q.shape[-2:]
    SK = K.shape[-2]
    BH = int(np.prod(Q.shape[:-2])) if Q.ndim > 2 else 1
    assert K.shape[-1] == D and V.shape == K.shape
    O = np.empty(Q.shape, np.float16)
    check(load().hexcuda_host_attn_f16(_p(Q), _p(K), _p(V), _p(O), BH, SQ, SK, D, scale,
                                       int(bool(causal))))
    return O


def online_softmax_step_f16(scores, V, running_max, running_sum, acc):
    """Returns the updated (running_max, running_sum, acc)."""
    scores, V = _c(scores, np.float16), _c(V, np.float16)
    acc = np.array(acc, np.float16, copy=True)
    BLK, D = V.shape
    m = np.array([running_max], np.float16)
    s = np.array([running_sum], np.float16)
    check(load().hexcuda_host_online_softmax_step_f16(_p(scores), _p(V), _p(m), _p(s), _p(acc),
                                                      BLK, D))
    return m[0], s[0], acc


# ------------------------------------------------------------ row operators

def softmax(x) -> np.ndarray:
    x = np.ascontiguousarray(x)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    if x.dtype == np.float32:
        check(load().hexcuda_host_softmax_f32(_p(x), _p(out), R, Cc))
    elif x.dtype == np.float16:
        check(load().hexcuda_host_softmax_f16(_p(x), _p(out), R, Cc))
    else:
        raise TypeError(x.dtype)
    return out


def layernorm(x, gamma, beta, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    gamma, beta = _c(gamma, x.dtype), _c(beta, x.dtype)
    out = np.empty_like(x)
    fn = {np.float32: load().hexcuda_host_layernorm_f32,
          np.float16: load().hexcuda_host_layernorm_f16}[x.dtype.type]
    check(fn(_p(x), _p(gamma), _p(beta), _p(out), R, Cc, eps))
    return out


def rmsnorm_f16(x, gamma, eps: float) -> np.ndarray:
    x, gamma = _c(x, np.float16), _c(gamma, np.float16)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    check(load().hexcuda_host_rmsnorm_f16(_p(x), _p(gamma), _p(out), R, Cc, eps))
    return out


def rmsnorm_gain_f16(x, gain, eps: float) -> np.ndarray:
    """RMS norm of each row of x [R, C] times one gain per row (fp16)."""
    x, gain = _c(x, np.float16), _c(gain, np.float16)
    R, Cc = x.shape
    out = np.empty_like(x)
    check(load().hexcuda_host_rmsnorm_gain_f16(_p(x), _p(gain), _p(out), R, Cc, eps))
    return out


def rowreduce(x, op: int) -> np.ndarray:
    """op 0 = row sum, op 1 = row max; fp32."""
    x = _c(x, np.float32)
    R, Cc = x.reshape(-1, x.shape[-1]).shape
    out = np.empty(R, np.float32)
    check(load().hexcuda_host_rowreduce_f32(_p(x), _p(out), R, Cc, op))
    return out
