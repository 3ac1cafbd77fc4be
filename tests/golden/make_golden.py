"""Generate the golden vectors in tests/golden/ from the reference's own code.

Run in a container where the hexkernels reference tree is mounted (default
/root/reference, override with HEXKERNELS_REF).  It builds the reference's
scalar reference.c files into oracle/_ref/libhexref.so (oracle/Makefile target
`ref`), regenerates each expert harness's inputs with the harness's own LCG
recipe (seed, value map, planted edge cases, parameter sweep), calls the
REFERENCE implementation on them and stores inputs + expected outputs as
compressed .npz files.  Large-shape cases draw inputs from
numpy.random.default_rng(seed) with the value distributions of the benchmark
configurations.

The fixtures are committed; the GPU box never runs this script.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import base64
import ctypes as C
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF_ROOT = Path(os.environ.get("HEXKERNELS_REF", "/root/reference"))

P = C.c_void_p


def lcg_stream(seed: int):
    s = seed & 0xFFFFFFFF
    while True:
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        yield s


def i8_top_byte(v: int) -> int:
    """(int8_t)(lcg >> 24)"""
    b = v >> 24
    return b - 256 if b >= 128 else b


def ptr(a: np.ndarray):
    return a.ctypes.data_as(P)


def load_ref():
    subprocess.run(["make", "-s", "-C", str(REPO / "oracle"), "ref",
                    f"REF_ROOT={REF_ROOT}"], check=True)
    return C.CDLL(str(REPO / "oracle" / "_ref" / "libhexref.so"))


def save(name: str, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz: " + ", ".join(f"{k}{list(v.shape)}" for k, v in arrays.items()))


# ----------------------------------------------------------------- integer

def gen_i8_gemm_requant(ref):
    # kernels/expert/i8_gemm_requant/harness.c:3-35 (M 32, N 32, K 66,
    # seed 0xA3C7F1, edges A[0]=127 B[0]=127 A[1]=-128 B[N]=127,
    # (mult, shift, zp) sets (3,4,0) and (1,0,0)).
    M, N, K = 32, 32, 66
    g = lcg_stream(0xA3C7F1)
    A = np.array([i8_top_byte(next(g)) for _ in range(M * K)], np.int8)
    B = np.array([i8_top_byte(next(g)) for _ in range(K * N)], np.int8)
    A[0], B[0], A[1], B[N] = 127, 127, -128, 127
    params = np.array([[3, 4, 0], [1, 0, 0]], np.int64)
    outs = []
    f = ref.ref_i8_gemm_requant
    for mult, shift, zp in params:
        out = np.full(M * N, -91, np.int8)
        f(ptr(A), ptr(B), ptr(out), M, N, K, C.c_int32(int(mult)), C.c_int(int(shift)),
          C.c_int8(int(zp)))
        outs.append(out.copy())
    save("i8_gemm_requant_harness", A=A, B=B, dims=np.array([M, N, K]), params=params,
         out=np.stack(outs))


def gen_i8_gemm_requant_256(ref):
    # Benchmark configuration: int8 x int8 -> int32 GEMM M=N=K=256, uniform
    # int8, mult in [2^30, 2^31), shift 8..15, seed 0.  That requant saturates
    # almost everywhere, so the fixture adds a non-saturating sweep (shift
    # 36..44, zp -3..3) that exercises rounding, plus small-mult cases.
    M = N = K = 256
    rng = np.random.default_rng(0)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    mult0 = int(rng.integers(2**30, 2**31))
    shift0 = int(rng.integers(8, 16))
    params = [[mult0, shift0, 0]]
    for shift in (36, 38, 40, 42, 44):
        params.append([int(rng.integers(2**30, 2**31)), shift, int(rng.integers(-3, 4))])
    params += [[1, 0, 0], [3, 4, -7], [-5, 9, 11], [2**31 - 1, 62, 0], [1234567, 30, 0]]
    params = np.array(params, np.int64)
    outs = []
    for mult, shift, zp in params:
        out = np.full(M * N, -91, np.int8)
        ref.ref_i8_gemm_requant(ptr(A), ptr(B), ptr(out), M, N, K, C.c_int32(int(mult)),
                                C.c_int(int(shift)), C.c_int8(int(zp)))
        outs.append(out.reshape(M, N).copy())
    save("i8_gemm_requant_256", A=A, B=B, params=params, out=np.stack(outs))


def gen_i8_gemm_bias_requant(ref):
    # kernels/expert/i8_gemm_bias_requant/harness.c:3-48 (32^3, seed 0xC9D4E2,
    # bias = (lcg & 0xFFFF) - 0x8000, edges incl. bias[0] = -2e6, bias[1] = 2e6).
    M = N = K = 32
    g = lcg_stream(0xC9D4E2)
    A = np.array([i8_top_byte(next(g)) for _ in range(M * K)], np.int8)
    B = np.array([i8_top_byte(next(g)) for _ in range(K * N)], np.int8)
    bias = np.array([(next(g) & 0xFFFF) - 0x8000 for _ in range(N)], np.int32)
    A[0], B[0], A[1], B[N] = 127, 127, -128, 127
    bias[0], bias[1], bias[2] = -2000000, 2000000, 0
    params = np.array([[3, 4, 0], [1, 0, 0], [1 << 20, 28, 5]], np.int64)
    outs = []
    for mult, shift, zp in params:
        out = np.full(M * N, -91, np.int8)
        ref.ref_i8_gemm_bias_requant(ptr(A), ptr(B), ptr(bias), ptr(out), M, N, K,
                                     C.c_int32(int(mult)), C.c_int(int(shift)),
                                     C.c_int8(int(zp)))
        outs.append(out.copy())
    save("i8_gemm_bias_requant_harness", A=A, B=B, bias=bias, dims=np.array([M, N, K]),
         params=params, out=np.stack(outs))


def gen_gemm_tile_zp_i8(ref):
    # kernels/expert/gemm_tile_zp_i8/harness.c:3-64 (M 8, N 8, K 94 with a
    # K tail, seed 0x3B77F210, (zpA, mult, shift) = (0,3,7), (-10,5,4), (20,1,0)).
    M, N, K = 8, 8, 94
    g = lcg_stream(0x3B77F210)
    A = np.array([i8_top_byte(next(g)) for _ in range(M * K)], np.int8)
    B = np.array([i8_top_byte(next(g)) for _ in range(K * N)], np.int8)
    A[0], B[0], A[1], B[N] = 127, 127, -128, 127
    for i in range(M):
        A[i * K + 92], A[i * K + 93] = 100, -50
    for j in range(N):
        B[92 * N + j], B[93 * N + j] = -80, 60
    params = np.array([[0, 3, 7], [-10, 5, 4], [20, 1, 0]], np.int64)
    outs = []
    for zpa, mult, shift in params:
        out = np.full(M * N, -91, np.int8)
        ref.ref_gemm_tile_zp_i8(ptr(A), ptr(B), ptr(out), M, N, K, C.c_int32(int(zpa)),
                                C.c_int32(int(mult)), C.c_int(int(shift)))
        outs.append(out.copy())
    save("gemm_tile_zp_i8_harness", A=A, B=B, dims=np.array([M, N, K]), params=params,
         out=np.stack(outs))


def gen_requant_per_channel(ref):
    # kernels/expert/requant_per_channel/harness.c:4-75 (R 40, C 25, seed
    # 0xBEEF77, a = (int32)lcg % 601 - 300 with C's truncating %, 5 sets).
    R, Cc = 40, 25
    g = lcg_stream(0xBEEF77)
    a = []
    for _ in range(R * Cc):
        v = next(g)
        v = v - (1 << 32) if v >= (1 << 31) else v
        r = abs(v) % 601
        a.append((r if v >= 0 else -r) - 300)
    a = np.array(a, np.int32)
    a[:5] = [4, -4, 300, -300, 0]
    mult_sets = np.array([
        [5, 5, 5, -3, 127] + [5] * 35,
        [13] * 40,
        [7, -7] * 20,
        [1, 2, 3, 4] * 10,
        [1, 2, 4, 8, 16] * 8,
    ], np.int32)
    shift_sets = np.array([
        [3, 0, 7, 2, 4] + [3] * 35,
        [7] * 40,
        [3] * 40,
        [0, 1, 2, 3] * 10,
        [0, 1, 2, 3, 4] * 8,
    ], np.int32)
    zps = np.array([0, -5, 0, 10, 0], np.int8)
    outs = []
    for k in range(5):
        out = np.full(R * Cc, -91, np.int8)
        m = np.ascontiguousarray(mult_sets[k])
        s = np.ascontiguousarray(shift_sets[k])
        ref.ref_requant_per_channel(ptr(a), ptr(out), R, Cc, ptr(m), ptr(s), C.c_int8(int(zps[k])))
        outs.append(out.copy())
    save("requant_per_channel_harness", a=a, dims=np.array([R, Cc]), mult=mult_sets,
         shift=shift_sets, zp=zps, out=np.stack(outs))


def gen_requantize_i32_u8(ref):
    # kernels/expert/requantize_i32_u8_dma/harness.c:18-77: N 262144,
    # a[i] = ((i*2731 + 5) & 0xFFFF) - 32768, edges a[0..5], MULT 5, SHIFT 8,
    # ZP 128; plus two more (mult, shift, zp) sets over the same input.
    n = 262144
    i = np.arange(n, dtype=np.int64)
    a = (((i * 2731 + 5) & 0xFFFF) - 32768).astype(np.int32)
    a[:6] = [32767, -32768, 0, 6400, 13000, -13000]
    params = np.array([[5, 8, 128], [-3, 2, 17], [40000, 20, 255]], np.int64)
    outs = []
    for mult, shift, zp in params:
        out = np.full(n, 0xA5, np.uint8)
        ref.ref_requantize_i32_u8_dma(ptr(a), ptr(out), n, C.c_int32(int(mult)),
                                      C.c_int(int(shift)), C.c_uint8(int(zp)))
        outs.append(out.copy())
    save("requantize_i32_u8_harness", params=params, out=np.stack(outs))


def gen_gemm_u8s8_pc(ref):
    # Composed u8 x s8 per-channel GEMM at a small shape with the benchmark's
    # value distributions (A u8, zpA 128, B s8, bias N(0,1000), mult in
    # [2^30, 2^31), shift spread so outputs cover [0, 255], zp_out 128).  The
    # int32 accumulator rawdot - zpA*colsum is exact integer arithmetic
    # (numpy int64, no overflow at these sizes); the per-channel requant and u8
    # saturation run through the reference's own requantize_i32_u8_dma
    # reference.c, one output column (channel) at a time.
    rng = np.random.default_rng(4)
    cases = []
    for (M, N, K) in [(64, 96, 160), (130, 72, 200)]:
        A = rng.integers(0, 256, size=(M, K), dtype=np.uint8)
        B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
        bias = np.round(rng.normal(0, 1000, size=N)).astype(np.int32)
        zpa = 128
        mult = rng.integers(2**30, 2**31, size=N, dtype=np.int64).astype(np.int32)
        acc = A.astype(np.int64) @ B.astype(np.int64) - zpa * B.astype(np.int64).sum(0)
        biased = acc + bias
        sigma = max(float(np.std(biased)), 1.0)
        # shift so that sigma * mult / 2^shift ~ 48
        shift = np.clip(np.round(np.log2(sigma * mult.astype(np.float64) / 48.0)), 0, 62).astype(np.int32)
        shift[0] = 0          # saturating channel
        shift[1] = 62         # all-zero channel (before zp)
        zp_out = 128
        out = np.zeros((M, N), np.uint8)
        col = np.zeros(M, np.uint8)
        for j in range(N):
            bj = np.ascontiguousarray(biased[:, j].astype(np.int32))
            ref.ref_requantize_i32_u8_dma(ptr(bj), ptr(col), M, C.c_int32(int(mult[j])),
                                          C.c_int(int(shift[j])), C.c_uint8(zp_out))
            out[:, j] = col
        cases.append(dict(A=A, B=B, bias=bias, mult=mult, shift=shift, zpa=np.int32(zpa),
                          zp_out=np.uint8(zp_out), out=out))
    arrays = {}
    for ci, c in enumerate(cases):
        for k, v in c.items():
            arrays[f"c{ci}_{k}"] = np.asarray(v)
    arrays["ncases"] = np.array(len(cases))
    save("gemm_u8s8_pc_small", **arrays)


def gen_hmx(ref):
    # The six HMX-convention u8 x s8 bundles.  Harness cases regenerate each
    # harness.c's inputs (hvx_lcg seed, value map, planted bias edges):
    #   hmx_matmul_i8_requant/harness.c:14-18   N 32, seed 0xC4F8, A %16, B %9-4
    #   hmx_matmul_i8_zp/harness.c:18-21        N 32, seed 0x2E90, A %8, B %7-3, zp 2
    #   i8_gemm_bias_relu_requant_hmx/harness.c:24-31
    #                                           N 64, seed 0xA6F7, A %8, B %7-3,
    #                                           bias %4001-2000, bias[0..2] = -2000, 2000, 0
    #   hmx_matmul_i8_64/harness.c:13-16        N 64, seed 0x8B22, A %8, B %7-3
    #   hmx_matmul_i8_deepk/harness.c:14-17     N 32, K 128, seed 0xD5A9, A %4, B %3-1
    #   hmx_matmul_i8_transposeB/harness.c:17-20 N 32, seed 0x7B21, A %8, Bt %7-3
    # Wide cases use full-range u8 / s8 inputs (|acc| well past the 12-bit
    # field, so the sx12 wrap is exercised) at n not a multiple of the GEMM
    # tile; products stay inside int32 there, so the reference is well defined.
    def lcg_mod(g, n, mod, off, dtype):
        return np.array([(next(g) % mod) - off for _ in range(n)], np.int64).astype(dtype)

    arrays = {}

    def run(tag, fn, A, B, extra_pre, out, *tail):
        getattr(ref, fn)(ptr(A), ptr(B), *extra_pre, ptr(out), *tail)
        arrays[f"{tag}_A"], arrays[f"{tag}_B"], arrays[f"{tag}_out"] = A, B, out

    n = 32
    g = lcg_stream(0xC4F8)
    A = lcg_mod(g, n * n, 16, 0, np.uint8); B = lcg_mod(g, n * n, 9, 4, np.int8)
    run("requant", "ref_hmx_matmul_i8_requant", A, B, [], np.full(n * n, 0x5A, np.int8), n)
    g = lcg_stream(0x2E90)
    A = lcg_mod(g, n * n, 8, 0, np.uint8); B = lcg_mod(g, n * n, 7, 3, np.int8)
    arrays["zp_zp"] = np.int32(2)
    run("zp", "ref_hmx_matmul_i8_zp", A, B, [C.c_int(2)], np.zeros(n * n, np.int32), n)
    n = 64
    g = lcg_stream(0xA6F7)
    A = lcg_mod(g, n * n, 8, 0, np.uint8); B = lcg_mod(g, n * n, 7, 3, np.int8)
    bias = lcg_mod(g, n, 4001, 2000, np.int32)
    bias[0], bias[1], bias[2] = -2000, 2000, 0
    arrays["bias_relu_bias"] = bias
    run("bias_relu", "ref_i8_gemm_bias_relu_requant_hmx", A, B, [ptr(bias)],
        np.zeros(n * n, np.uint8), n)
    g = lcg_stream(0x8B22)
    A = lcg_mod(g, n * n, 8, 0, np.uint8); B = lcg_mod(g, n * n, 7, 3, np.int8)
    run("i64", "ref_hmx_matmul_i8_64", A, B, [], np.zeros(n * n, np.int32), n)
    n, K = 32, 128
    g = lcg_stream(0xD5A9)
    A = lcg_mod(g, n * K, 4, 0, np.uint8); B = lcg_mod(g, K * n, 3, 1, np.int8)
    arrays["deepk_K"] = np.int32(K)
    run("deepk", "ref_hmx_matmul_i8_deepk", A, B, [], np.zeros(n * n, np.int32), n, K)
    n = 32
    g = lcg_stream(0x7B21)
    A = lcg_mod(g, n * n, 8, 0, np.uint8); B = lcg_mod(g, n * n, 7, 3, np.int8)
    run("transposeB", "ref_hmx_matmul_i8_transposeB", A, B, [], np.zeros(n * n, np.int32), n)

    # wide, full-range cases
    rng = np.random.default_rng(11)
    u8 = lambda k: rng.integers(0, 256, size=k, dtype=np.uint8)
    s8 = lambda k: rng.integers(-128, 128, size=k, dtype=np.int8)
    n = 160
    run("w_requant", "ref_hmx_matmul_i8_requant", u8(n * n), s8(n * n), [],
        np.zeros(n * n, np.int8), n)
    n = 144
    arrays["w_zp_zp"] = np.int32(131)
    run("w_zp", "ref_hmx_matmul_i8_zp", u8(n * n), s8(n * n), [C.c_int(131)],
        np.zeros(n * n, np.int32), n)
    n = 200
    wb = rng.integers(-3000, 3001, size=n, dtype=np.int32)
    arrays["w_bias_relu_bias"] = wb
    run("w_bias_relu", "ref_i8_gemm_bias_relu_requant_hmx", u8(n * n), s8(n * n), [ptr(wb)],
        np.zeros(n * n, np.uint8), n)
    n, K = 136, 1000
    arrays["w_deepk_K"] = np.int32(K)
    run("w_deepk", "ref_hmx_matmul_i8_deepk", u8(n * K), s8(K * n), [],
        np.zeros(n * n, np.int32), n, K)
    n = 130
    run("w_transposeB", "ref_hmx_matmul_i8_transposeB", u8(n * n), s8(n * n), [],
        np.zeros(n * n, np.int32), n)
    save("hmx_gemm", **arrays)


def gen_hmx_family(ref):
    # The 24 HMX-convention bundles of tests/hmx_family.py, each run through
    # its own reference.c on seeded inputs: full-range u8 / s8 operands at
    # sizes that are not multiples of the GEMM tile (products stay inside
    # int32, so the references are well defined), small operands where a
    # 256-entry table is indexed by the result.
    sys.path.insert(0, str(HERE.parent))
    from hmx_family import BUNDLES, OUT_DTYPE, shape_of
    rng = np.random.default_rng(23)
    arrays = {}
    for b, (params, kw) in BUNDLES.items():
        M, N, K = shape_of(b)
        small = "lut" in kw["store"]
        a = {
            "A": (rng.integers(0, 4, M * K) if small else rng.integers(0, 256, M * K)).astype(np.uint8),
            "bias": rng.integers(-200 if small else -3000, 201 if small else 3001, N).astype(np.int32),
            "res32": rng.integers(-10**6, 10**6, M * N).astype(np.int32),
            "res8": rng.integers(-128, 128, M * N).astype(np.int8),
            "lut32": rng.integers(-10**5, 10**5, 256).astype(np.int32),
            "lut8": rng.integers(-128, 128, 256).astype(np.int8),
        }
        bvals = rng.integers(-1, 2, K * N) if small else rng.integers(-128, 128, K * N)
        a["B"] = a["Bt"] = a["x"] = bvals.astype(np.int8)
        out = np.zeros(M * N, OUT_DTYPE[kw["store"]])
        args = []
        for prm in params:
            if prm == "out":
                args.append(ptr(out))
            elif prm in ("n", "M"):
                args.append(M)
            elif prm == "N":
                args.append(N)
            elif prm == "K":
                args.append(K)
            else:
                args.append(ptr(a[prm]))
        getattr(ref, "ref_" + b)(*args)
        for prm in params:
            if prm in a:
                arrays[f"{b}__{prm}"] = a[prm]
        arrays[f"{b}__out"] = out
        arrays[f"{b}__mnk"] = np.array([M, N, K], np.int32)
    save("hmx_family", **arrays)


def gen_requant_family(ref):
    # The elementwise requant bundles of tests/requant_family.py plus
    # epilogue_bias_i32 / epilogue_relu_i8, run through their own reference.c
    # on seeded inputs (n = 1037, not a multiple of the 16-element vector
    # step), three parameter sets each where the bundle takes parameters
    # (large mult / shift, a small mult, a negative mult).  Inputs are sized so
    # every int64 product stays inside int64, where the references are defined.
    sys.path.insert(0, str(HERE.parent))
    from requant_family import RQ_BUNDLES
    rng = np.random.default_rng(31)
    n = 1037
    arrays = {}
    for b, (params, kw) in RQ_BUNDLES.items():
        sets = [(int(rng.integers(2**30, 2**31)), int(rng.integers(30, 41)), int(rng.integers(-20, 21))),
                (3, 4, -2), (-123457, 12, 3)] if "mult" in params else [(0, 0, 0), (0, 0, 0)]
        for ci, (mult, shift, zp) in enumerate(sets):
            big = 2**20 if kw.get("pre") == "mul_add" else 2**30
            a = {"a32": rng.integers(-big, big, n).astype(np.int32),
                 "b32": rng.integers(-big, big, n).astype(np.int32),
                 "a8": rng.integers(-128, 128, n).astype(np.int8),
                 "b8": rng.integers(-128, 128, n).astype(np.int8),
                 "lut": rng.integers(-128, 128, 256).astype(np.int8)}
            if "mult" not in params:
                a["a32"] = rng.integers(-3000, 3000, n).astype(np.int32)
            lo, hi = sorted(int(v) for v in rng.integers(-100, 100, 2))
            out = np.zeros(n, np.int8)
            args = []
            for prm in params:
                if prm == "out":
                    args.append(ptr(out))
                elif prm == "n":
                    args.append(n)
                elif prm == "mult":
                    args.append(C.c_int32(mult))
                elif prm == "shift":
                    args.append(C.c_int(shift))
                elif prm == "zp":
                    args.append(C.c_int8(zp))
                elif prm == "lo":
                    args.append(C.c_int8(lo))
                elif prm == "hi":
                    args.append(C.c_int8(hi))
                else:
                    args.append(ptr(a[prm]))
            getattr(ref, "ref_" + b)(*args)
            key = f"{b}__c{ci}__"
            for prm in params:
                if prm in a:
                    arrays[key + prm] = a[prm]
            arrays.update({key + "out": out, key + "mult": np.int32(mult), key + "shift": np.int32(shift),
                           key + "zp": np.int32(zp), key + "lo": np.int32(lo), key + "hi": np.int32(hi)})
    R, Cc = 37, 300
    acc = rng.integers(-2**31, 2**31, (R, Cc), dtype=np.int64).astype(np.int32)
    bias = rng.integers(-2**31, 2**31, Cc, dtype=np.int64).astype(np.int32)
    outb = np.zeros((R, Cc), np.int32)
    ref.ref_epilogue_bias_i32(ptr(acc), ptr(bias), ptr(outb), R, Cc)
    x8 = rng.integers(-128, 128, n).astype(np.int8)
    outr = np.zeros(n, np.int8)
    ref.ref_epilogue_relu_i8(ptr(x8), ptr(outr), n)
    arrays.update({"epilogue_bias_i32__acc": acc, "epilogue_bias_i32__bias": bias,
                   "epilogue_bias_i32__out": outb, "epilogue_relu_i8__x": x8,
                   "epilogue_relu_i8__out": outr})
    save("requant_family", **arrays)


def gen_int8_attention_hmx(ref):
    # i8_attention_qkt_hmx / _av_hmx at S = 72, D = 40 (off the tile grid),
    # i8_attention_qkt_av_hmx at S = 32 (its reference keeps Sc in a 32x32
    # array), D = 72, i8_gqa_qkt_hmx at its fixed shape (2 query heads, 1 KV
    # head, S = D = 64); full-range u8 / s8 inputs, reference.c outputs.
    rng = np.random.default_rng(41)
    u8 = lambda k: rng.integers(0, 256, k, dtype=np.uint8)
    s8 = lambda k: rng.integers(-128, 128, k, dtype=np.int8)
    S, D = 72, 40
    q, k = u8(S * D), s8(S * D)
    o = np.zeros(S * S, np.uint16)
    ref.ref_i8_attention_qkt_hmx(ptr(q), ptr(k), ptr(o), S, D)
    arrays = {"qkt_Q": q, "qkt_K": k, "qkt_out": o, "qkt_SD": np.array([S, D], np.int32)}
    pm, v = u8(S * S), s8(S * D)
    o = np.zeros(S * D, np.uint16)
    ref.ref_i8_attention_av_hmx(ptr(pm), ptr(v), ptr(o), S, D)
    arrays.update({"av_P": pm, "av_V": v, "av_out": o, "av_SD": np.array([S, D], np.int32)})
    S, D = 32, 72
    q, k, v = u8(S * D), s8(S * D), s8(S * D)
    o = np.zeros(S * D, np.int32)
    ref.ref_i8_attention_qkt_av_hmx(ptr(q), ptr(k), ptr(v), ptr(o), S, D)
    arrays.update({"qkav_Q": q, "qkav_K": k, "qkav_V": v, "qkav_out": o,
                   "qkav_SD": np.array([S, D], np.int32)})
    q, k = u8(2 * 64 * 64), s8(64 * 64)
    o = np.zeros(2 * 64 * 64, np.uint16)
    ref.ref_i8_gqa_qkt_hmx(ptr(q), ptr(k), ptr(o))
    arrays.update({"gqa_Q": q, "gqa_K": k, "gqa_out": o})
    save("int8_attention_hmx", **arrays)


def gen_int8_attention_blocks(ref):
    # gqa_attention (fixed 4 query / 2 KV heads, SEQ 8, D 16), i8_attention_block
    # (S 48, D 40), i8_gqa_attention_block (fixed 2 / 1 heads, S = D = 64),
    # i8_rope_attention_block (S 40, D 56), i8_decoder_block (S 24, D 40,
    # Dff 100), each through its reference.c on seeded inputs; the exp table is
    # round(255 exp((i - 255) / 24)), the other tables are seeded int8.
    rng = np.random.default_rng(53)
    exp_lut = np.round(255 * np.exp((np.arange(256) - 255) / 24.0)).astype(np.uint8)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    u8 = lambda *sh: rng.integers(0, 256, sh, dtype=np.uint8)
    a = {"exp_lut": exp_lut}
    q, k, v = s8(4, 8, 16), s8(2, 8, 16), s8(2, 8, 16)
    o = np.zeros((4, 8, 16), np.int8)
    ref.ref_gqa_attention(ptr(q), ptr(k), ptr(v), ptr(exp_lut), ptr(o), C.c_int32(1 << 30), 41,
                          C.c_int32(1 << 30), 41)
    a.update(gqa_Q=q, gqa_K=k, gqa_V=v, gqa_out=o)
    S, D = 48, 40
    q, k, v = u8(S, D), s8(S, D), s8(S, D)
    o = np.zeros((S, D), np.uint16)
    ref.ref_i8_attention_block(ptr(q), ptr(k), ptr(v), ptr(o), S, D, ptr(exp_lut))
    a.update(blk_Q=q, blk_K=k, blk_V=v, blk_out=o)
    q, k, v = u8(2, 64, 64), s8(1, 64, 64), s8(1, 64, 64)
    o = np.zeros((2, 64, 64), np.uint16)
    ref.ref_i8_gqa_attention_block(ptr(q), ptr(k), ptr(v), ptr(o), ptr(exp_lut))
    a.update(gblk_Q=q, gblk_K=k, gblk_V=v, gblk_out=o)
    S, D = 40, 56
    q, k, v = u8(S, D), s8(S, D), s8(S, D)
    cs = rng.integers(-64, 65, (S, D // 2)).astype(np.int8)
    sn = rng.integers(-64, 65, (S, D // 2)).astype(np.int8)
    o = np.zeros((S, D), np.uint16)
    ref.ref_i8_rope_attention_block(ptr(q), ptr(k), ptr(v), ptr(cs), ptr(sn), ptr(o), S, D, 6,
                                    ptr(exp_lut))
    a.update(rope_Q=q, rope_K=k, rope_V=v, rope_cos=cs, rope_sin=sn, rope_out=o)
    S, D, F = 24, 40, 100
    x = rng.integers(0, 64, (S, D), dtype=np.uint8)
    w1, w2 = s8(D, F), s8(F, D)
    b1 = rng.integers(-200, 200, F).astype(np.int32)
    b2 = rng.integers(-50, 50, D).astype(np.int32)
    act = s8(256)
    o = np.zeros((S, D), np.int8)
    ref.ref_i8_decoder_block(ptr(x), ptr(w1), ptr(b1), ptr(act), ptr(w2), ptr(b2), ptr(exp_lut),
                             ptr(o), S, D, F)
    a.update(dec_X=x, dec_W1=w1, dec_b1=b1, dec_act=act, dec_W2=w2, dec_b2=b2, dec_out=o)
    for key, val in a.items():
        if key.endswith("_out"):
            assert len(np.unique(val)) > 8, key   # not a degenerate case
    save("int8_attention_blocks", **a)


def gen_f16_family(ref):
    # The fp16 post-op GEMM bundles through their reference.c at sizes off the
    # tile grid, inputs N(0,1)/sqrt(K) in fp16 (outputs of order 1; the GELU
    # and leaky cases see both signs).
    rng = np.random.default_rng(61)
    f16 = lambda *sh, k=1: (rng.standard_normal(sh) / np.sqrt(k)).astype(np.float16)
    a = {}
    n, kd = 72, 136

    def run(tag, fn, *args):
        getattr(ref, "ref_" + fn)(*args)

    for name, k in (("fp16_matmul_gelu_hmx", n), ("fp16_matmul_hmx_32x32", n), ("hmx_matmul_fp16_32", n),
                    ("hmx_matmul_fp16_relu", n), ("hmx_conv1x1_fp16", n)):
        A, B = f16(n, n, k=n), f16(n, n)
        o = np.zeros((n, n), np.float16)
        run(name, name, ptr(A), ptr(B), ptr(o), n)
        a.update({f"{name}__A": A, f"{name}__B": B, f"{name}__out": o})
    for name in ("fp16_matmul_hmx_deepk", "fp16_matmul_leaky_relu_hmx"):
        A, B = f16(n, kd, k=kd), f16(kd, n)
        o = np.zeros((n, n), np.float16)
        run(name, name, ptr(A), ptr(B), ptr(o), n, kd)
        a.update({f"{name}__A": A, f"{name}__B": B, f"{name}__out": o})
    A, B, bias = f16(n, n, k=n), f16(n, n), f16(n)
    o = np.zeros((n, n), np.float16)
    run("b", "hmx_matmul_fp16_bias", ptr(A), ptr(B), ptr(bias), ptr(o), n)
    a.update({"hmx_matmul_fp16_bias__A": A, "hmx_matmul_fp16_bias__B": B,
              "hmx_matmul_fp16_bias__bias": bias, "hmx_matmul_fp16_bias__out": o})
    A, B, c0 = f16(n, n, k=n), f16(n, n), f16(n, n)
    o = c0.copy()
    run("m", "hmx_tile_mac_fp16_32", ptr(A), ptr(B), ptr(o), n)
    a.update({"hmx_tile_mac_fp16_32__A": A, "hmx_tile_mac_fp16_32__B": B,
              "hmx_tile_mac_fp16_32__C": c0, "hmx_tile_mac_fp16_32__out": o})
    M, N, D = 60, 100, 40
    Q, K = f16(M, D, k=D), f16(D, N)
    o = np.zeros((M, N), np.float16)
    ref.ref_qkt_tile_fp16(ptr(Q), ptr(K), ptr(o), M, N, D, C.c_uint16(np.float16(0.125).view(np.uint16)))
    a.update({"qkt_tile_fp16__Q": Q, "qkt_tile_fp16__K": K, "qkt_tile_fp16__out": o})
    Am, V = f16(M, N, k=N), f16(D, N)
    o = np.zeros((M, D), np.float16)
    ref.ref_av_tile_fp16(ptr(Am), ptr(V), ptr(o), M, N, D)
    a.update({"av_tile_fp16__A": Am, "av_tile_fp16__V": V, "av_tile_fp16__out": o})
    # the callers that round the accumulator before their post-op
    for name in ("fp16_matmul_bias_gelu", "fp16_matmul_bias_relu"):
        A, B, bias = f16(n, kd, k=kd), f16(kd, n), f16(n)
        o = np.zeros((n, n), np.float16)
        run(name, name, ptr(A), ptr(B), ptr(bias), ptr(o), n, kd)
        a.update({f"{name}__A": A, f"{name}__B": B, f"{name}__bias": bias, f"{name}__out": o})
    A, B, c0 = f16(n, kd, k=kd), f16(kd, n), f16(n, n)
    o = np.zeros((n, n), np.float16)
    run("r", "fp16_matmul_residual", ptr(A), ptr(B), ptr(c0), ptr(o), n, kd)
    a.update({"fp16_matmul_residual__A": A, "fp16_matmul_residual__B": B,
              "fp16_matmul_residual__C": c0, "fp16_matmul_residual__out": o})
    for name in ("fp16_matmul_sigmoid", "fp16_matmul_tanh"):
        A, B = f16(n, kd, k=kd), f16(kd, n)
        o = np.zeros((n, n), np.float16)
        run(name, name, ptr(A), ptr(B), ptr(o), n, kd)
        a.update({f"{name}__A": A, f"{name}__B": B, f"{name}__out": o})
    A, B = f16(n, n, k=n), f16(n, n)
    o = np.zeros((n, n), np.float16)
    run("g", "ai_fp16_matmul_gelu", ptr(A), ptr(B), ptr(o), n)
    a.update({"ai_fp16_matmul_gelu__A": A, "ai_fp16_matmul_gelu__B": B, "ai_fp16_matmul_gelu__out": o})
    save("f16_family", **a)


def gen_i8_callers(ref):
    # Callers of the int8 GEMM + requant and HMX paths through their
    # reference.c: gemm_bias_relu_requant (70 x 90 x 150), i8_linear_relu_requant
    # and i8_matvec_bias_requant (300 x 520), hmx_conv1x1_i8 (n 72),
    # i8_gemm_tiled_bias_relu_requant (60 x 100 x 130), i8_conv2d_1x1_hmx and
    # i8_pointwise_conv_hmx (their fixed shapes); full-range operands.
    rng = np.random.default_rng(71)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    u8 = lambda *sh: rng.integers(0, 256, sh, dtype=np.uint8)
    a = {}
    M, N, K = 70, 90, 150
    A, B = s8(M, K), s8(K, N)
    bias = rng.integers(-40000, 40000, N).astype(np.int32)
    o = np.zeros((M, N), np.int8)
    ref.ref_gemm_bias_relu_requant(ptr(A), ptr(B), ptr(bias), ptr(o), M, N, K, C.c_int32(1 << 30), 38,
                                   C.c_int8(3))
    a.update(gbr_A=A, gbr_B=B, gbr_bias=bias, gbr_out=o)
    M, K = 300, 520
    A, x = s8(M, K), s8(K)
    bias = rng.integers(-40000, 40000, M).astype(np.int32)
    for name in ("i8_linear_relu_requant", "i8_matvec_bias_requant"):
        o = np.zeros(M, np.int8)
        getattr(ref, "ref_" + name)(ptr(A), ptr(x), ptr(bias), ptr(o), M, K, C.c_int32(1 << 30), 38,
                                    C.c_int8(-2))
        a[name + "_out"] = o
    a.update(mv_A=A, mv_x=x, mv_bias=bias)
    n = 72
    In, W = u8(n, n), s8(n, n)
    bias = rng.integers(-3000, 3000, n).astype(np.int32)
    o = np.zeros((n, n), np.int32)
    ref.ref_hmx_conv1x1_i8(ptr(In), ptr(W), ptr(bias), ptr(o), n)
    a.update(c11_In=In, c11_W=W, c11_bias=bias, c11_out=o)
    M, N, K = 60, 100, 130
    A, B = u8(M, K), s8(K, N)
    bias = rng.integers(-3000, 3000, N).astype(np.int32)
    o = np.zeros((M, N), np.uint8)
    ref.ref_i8_gemm_tiled_bias_relu_requant(ptr(A), ptr(B), ptr(bias), ptr(o), M, N, K)
    a.update(tbr_A=A, tbr_B=B, tbr_bias=bias, tbr_out=o)
    for name, cin in (("i8_conv2d_1x1_hmx", 64), ("i8_pointwise_conv_hmx", 96)):
        inp, W = u8(cin, 64), s8(64, cin)
        o = np.zeros((64, 64), np.uint16)
        getattr(ref, "ref_" + name)(ptr(inp), ptr(W), ptr(o), 64)
        a.update({name + "_in": inp, name + "_W": W, name + "_out": o})
    save("i8_callers", **a)


# ----------------------------------------------------------------- fp16

def gen_hf_q(g, mod, off, step):
    return np.array([((next(g) % mod) - off) * step], np.float16)[0]


def hf_array(seed_iter, n, mod, off, step):
    return np.array([((next(seed_iter) % mod) - off) * step for _ in range(n)],
                    np.float32).astype(np.float16)


def gen_f16_gemms(ref):
    # kernels/expert/fp16_attention_qkt_hmx/harness.c:10-33 (n 32, k_dim 128,
    # seed 0x9C412, values (lcg % 7 - 3) * 0.25, K stored [n, k_dim]).
    g = lcg_stream(0x9C412)
    n, kd = 32, 128
    Q = hf_array(g, n * kd, 7, 3, 0.25)
    K = hf_array(g, n * kd, 7, 3, 0.25)
    out = np.zeros(n * n, np.float16)
    ref.ref_fp16_attention_qkt_hmx(ptr(Q), ptr(K), ptr(out), n, kd)
    save("gemm_f16_nt_harness", A=Q, Bt=K, dims=np.array([n, n, kd]), out=out)

    # kernels/expert/hmx_matmul_fp16_deepk/harness.c (n 32, k_dim 128,
    # seed 0xC0FFEE) -- row-major B[k_dim][n].
    g = lcg_stream(0xC0FFEE)
    A = hf_array(g, n * kd, 7, 3, 0.25)
    B = hf_array(g, kd * n, 7, 3, 0.25)
    out = np.zeros(n * n, np.float16)
    ref.ref_hmx_matmul_fp16_deepk(ptr(A), ptr(B), ptr(out), n, kd)
    save("gemm_f16_nn_harness", A=A, B=B, dims=np.array([n, n, kd]), out=out)

    # kernels/expert/fp16_attention_av_hmx/harness.c (n 32, Skv 128, seed 0x5A17F)
    g = lcg_stream(0x5A17F)
    Pm = hf_array(g, n * kd, 7, 3, 0.25)
    V = hf_array(g, kd * n, 7, 3, 0.25)
    out = np.zeros(n * n, np.float16)
    ref.ref_fp16_attention_av_hmx(ptr(Pm), ptr(V), ptr(out), n, kd)
    save("attn_av_f16_harness", A=Pm, B=V, dims=np.array([n, n, kd]), out=out)

    # Multi-tile shapes with the benchmark distribution N(0,1)/sqrt(K) through
    # the same reference (square n x n output, any k_dim).
    rng = np.random.default_rng(3)
    for (n, kd) in [(256, 512), (192, 320)]:
        A = (rng.standard_normal((n, kd)) / np.sqrt(kd)).astype(np.float16)
        Bt = (rng.standard_normal((n, kd)) / np.sqrt(kd)).astype(np.float16)
        out = np.zeros((n, n), np.float16)
        ref.ref_fp16_attention_qkt_hmx(ptr(A), ptr(Bt), ptr(out), n, kd)
        save(f"gemm_f16_nt_{n}x{kd}", A=A, Bt=Bt, out=out)


def gen_flash_attention(ref):
    # kernels/expert/fp16_flash_attention_tile/harness.c:12-60 (SQ 16, SK 64,
    # DH 64, seed 0xF1A54A11, values (lcg % 9 - 4) * 0.25, Q row 0 and K row
    # SK-1 forced to 1.0 so the running max moves on the final tile).
    SQ, SK, DH = 16, 64, 64
    g = lcg_stream(0xF1A54A11)
    Q = hf_array(g, SQ * DH, 9, 4, 0.25)
    K = hf_array(g, SK * DH, 9, 4, 0.25)
    V = hf_array(g, SK * DH, 9, 4, 0.25)
    Q[:DH] = 1.0
    K[(SK - 1) * DH:] = 1.0
    O = np.zeros(SQ * DH, np.float16)
    ref.ref_fp16_flash_attention_tile(ptr(Q), ptr(K), ptr(V), ptr(O), SQ, SK, DH)
    save("flash_attn_tile_harness", Q=Q, K=K, V=V, dims=np.array([SQ, SK, DH]), O=O)

    # Larger non-causal tiles (the reference caps SK at 64) with N(0,1) inputs
    # and the reference's FLASH_SCALE of 0.125.
    rng = np.random.default_rng(5)
    for (SQ, SK, DH) in [(256, 64, 64), (200, 48, 128)]:
        Q = rng.standard_normal((SQ, DH)).astype(np.float16)
        K = rng.standard_normal((SK, DH)).astype(np.float16)
        V = rng.standard_normal((SK, DH)).astype(np.float16)
        O = np.zeros((SQ, DH), np.float16)
        ref.ref_fp16_flash_attention_tile(ptr(Q), ptr(K), ptr(V), ptr(O), SQ, SK, DH)
        save(f"flash_attn_{SQ}x{SK}x{DH}", Q=Q, K=K, V=V, O=O)


def gen_online_softmax_step(ref):
    # kernels/expert/online_softmax_step_fp16/harness.c:16-135: BLK 24, D 48,
    # three cases (init m, init l, init acc, seed, biased index, biased value).
    BLK, D = 24, 48
    cases = [(-30000.0, 0.0, 0.0, 0xA5C31, -1, 0.0),
             (1.0, 3.0, 0.5, 0xBEEF77, 3, 5.0),
             (20.0, 2.0, 1.5, 0xC0DE99, -1, 0.0)]
    arrays = {}
    for ci, (m0, l0, a0, seed, bi, bv) in enumerate(cases):
        g = lcg_stream(seed)
        scores = hf_array(g, BLK, 17, 8, 0.5)
        if bi >= 0:
            scores[bi] = bv
        V = hf_array(g, BLK * D, 9, 4, 0.5)
        rmax = np.array([m0], np.float16)
        rsum = np.array([l0], np.float16)
        acc = np.full(D, a0, np.float16)
        arrays[f"c{ci}_scores"], arrays[f"c{ci}_V"] = scores.copy(), V.copy()
        arrays[f"c{ci}_state_in"] = np.concatenate([rmax, rsum, acc])
        ref.ref_online_softmax_step_fp16(ptr(scores), ptr(V), ptr(rmax), ptr(rsum), ptr(acc),
                                         BLK, D)
        arrays[f"c{ci}_state_out"] = np.concatenate([rmax, rsum, acc])
    arrays["dims"] = np.array([BLK, D])
    save("online_softmax_step_harness", **arrays)


def gen_rows(ref):
    # kernels/expert/fp16_softmax/harness.c:4-36 (R 8, C 256, seed 0x50F7,
    # values (lcg % 13 - 6) * 0.5, row 0 one dominant max, row 1 uniform).
    R, Cc = 8, 256
    g = lcg_stream(0x50F7)
    x = hf_array(g, R * Cc, 13, 6, 0.5)
    x[:Cc] = -3.0
    x[7] = 3.0
    x[Cc:2 * Cc] = 1.0
    out = np.zeros(R * Cc, np.float16)
    ref.ref_fp16_softmax(ptr(x), ptr(out), R, Cc)
    save("softmax_f16_harness", x=x, dims=np.array([R, Cc]), out=out)

    # wider random fp16 softmax (the reference caps C at 256)
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((96, 256)) * 4).astype(np.float16)
    out = np.zeros((96, 256), np.float16)
    ref.ref_fp16_softmax(ptr(x), ptr(out), 96, 256)
    save("softmax_f16_96x256", x=x, out=out)

    # kernels/expert/fp16_layernorm/harness.c:4-43 (n 2048, seed 0x1A9E5,
    # gamma 1 + 0.25*((i%5)-2), beta 0.25*((i%7)-3), edges x[0]=3 x[1]=-3 x[n-1]=0)
    n = 2048
    g = lcg_stream(0x1A9E5)
    x = hf_array(g, n, 13, 6, 0.5)
    i = np.arange(n)
    gamma = (1.0 + 0.25 * ((i % 5) - 2)).astype(np.float16)
    beta = (0.25 * ((i % 7) - 3)).astype(np.float16)
    x[0], x[1], x[n - 1] = 3.0, -3.0, 0.0
    out = np.zeros(n, np.float16)
    ref.ref_fp16_layernorm(ptr(x), ptr(gamma), ptr(beta), ptr(out), n)
    save("layernorm_f16_harness", x=x, gamma=gamma, beta=beta, out=out)

    # kernels/expert/fp16_rmsnorm/harness.c (n 2048, same recipe without beta)
    rms_src = (REF_ROOT / "kernels/expert/fp16_rmsnorm/harness.c").read_text()
    seed = int(re.search(r"uint32_t s = (0x[0-9A-Fa-f]+)u", rms_src).group(1), 16)
    g = lcg_stream(seed)
    x = hf_array(g, n, 13, 6, 0.5)
    x[0], x[1], x[n - 1] = 3.0, -3.0, 0.0
    out = np.zeros(n, np.float16)
    ref.ref_fp16_rmsnorm(ptr(x), ptr(gamma), ptr(out), n)
    save("rmsnorm_f16_harness", x=x, gamma=gamma, out=out, seed=np.array(seed))


def gen_mined_fp32_sum():
    # kernels/mined/fp32_sum/harness.c: the torch-made golden embedded as
    # base64 (48 x 128 fp32 input) and its hex-float expected sum.
    src = (REF_ROOT / "kernels/mined/fp32_sum/harness.c").read_text()
    body = src.split("static const char b64_in_0[] =", 1)[1].split(";", 1)[0]
    b64 = "".join(re.findall(r'"([^"]*)"', body))
    x = np.frombuffer(base64.b64decode(b64), dtype=np.float32).copy()
    gold = re.search(r"golden_out_0\[1\][^=]*=\s*\{\s*([^}]+)\}", src).group(1).strip()
    exp = np.float32(float.fromhex(gold.rstrip("f")))
    knu = re.search(r"forge2_close_acc\([^;]*?accum_s_0\[i\],\s*([^,]+),", src).group(1)
    save("rowsum_fp32_mined", x=x, out=np.array([exp], np.float32),
         knu=np.array([float.fromhex(knu.strip().rstrip("f"))], np.float32))


def gen_reduce_family(ref):
    # The integer reduction bundles of tests/reduce_family.py run through
    # their own reference.c on seeded full-range inputs (vtcm_reduce_i32:
    # |a| < 2^18, so the reference's signed int32 sum stays defined), four
    # sizes each (1, 17, 1000 and 4099 elements; g = 1, 17, 250 and 1025
    # groups for the 4-wide group sum), the arg reductions with their
    # extreme planted at three positions; gqa_group_reduce_i8 on three
    # shapes (H, G, M, N) = (8, 2, 5, 33), (12, 3, 4, 16), (7, 2, 3, 3).
    sys.path.insert(0, str(HERE.parent))
    from reduce_family import RD_BUNDLES, ctypes_args, make_inputs, out_buffer
    rng = np.random.default_rng(83)
    arrays = {}
    for b, (params, dt, kind) in RD_BUNDLES.items():
        if kind[0] == "gqa":
            cases = []
            for H, G, M, N in ((8, 2, 5, 33), (12, 3, 4, 16), (7, 2, 3, 3)):
                arr = make_inputs(b, rng, 0)
                arr.update(H=H, G=G, M=M, N=N,
                           X=rng.integers(-128, 128, H * M * N).astype(np.int8))
                cases.append(arr)
        else:
            sizes = (4, 68, 1000, 4100) if kind[0] == "group_sum" else (1, 17, 1000, 4099)
            cases = [make_inputs(b, rng, n) for n in sizes]
        for ci, arr in enumerate(cases):
            out = out_buffer(b, arr)
            getattr(ref, "ref_" + b)(*ctypes_args(b, arr, out))
            key = f"{b}__c{ci}__"
            for k, v in arr.items():
                arrays[key + k] = np.asarray(v)
            arrays[key + "out"] = out
    save("reduce_family", **arrays)


def gen_i8_acc_callers(ref):
    # The raw-accumulator int8 GEMM callers, the requant + residual GEMM and
    # the two-layer FFN through their reference.c at shapes off the tile
    # grid: full-range operands where the bundle saturates or keeps int32,
    # small-range operands (|x| <= 4) where a table or the int8 range must be
    # hit inside its range; ffn_relu_block at its reference's fixed hidden
    # buffer (M * V <= 256).
    rng = np.random.default_rng(97)
    s8 = lambda lo, hi, *sh: rng.integers(lo, hi, sh, dtype=np.int8)
    a = {}

    def run(name, args, **arrs):
        getattr(ref, "ref_" + name)(*args)
        for k, v in arrs.items():
            a[f"{name}__{k}"] = v

    for name, (M, N, K), bt in (("gemm_tile_i8", (70, 130, 200), True),
                                ("gemm_tile_deepk_i8", (40, 70, 1100), False),
                                ("i8_gemm_tile", (129, 65, 77), False)):
        A, B = s8(-128, 128, M, K), s8(-128, 128, *((N, K) if bt else (K, N)))
        C_ = np.zeros((M, N), np.int32)
        run(name, (ptr(A), ptr(B), ptr(C_), M, N, K), A=A, B=B, out=C_)
    M, N, K = 100, 90, 300
    A, B = s8(-128, 128, M, K), s8(-128, 128, K, N)
    bias = rng.integers(-2**20, 2**20, N).astype(np.int32)
    C_ = np.zeros((M, N), np.int32)
    run("i8_gemm_bias", (ptr(A), ptr(B), ptr(bias), ptr(C_), M, N, K), A=A, B=B, bias=bias, out=C_)
    M, N, K = 33, 40, 50
    A, B = s8(-128, 128, 4, M, K), s8(-128, 128, 4, K, N)
    bias = rng.integers(-50000, 50000, (4, N)).astype(np.int32)
    C0, C1 = np.zeros((4, M, N), np.int32), np.zeros((4, M, N), np.int32)
    run("i8_batch_matmul", (ptr(A), ptr(B), ptr(C0), M, N, K), A=A, B=B, out=C0)
    run("i8_batch_matmul_bias", (ptr(A), ptr(B), ptr(bias), ptr(C1), M, N, K), bias=bias, out=C1)
    M, N, K = 64, 80, 96
    A, B = s8(-4, 5, M, K), s8(-4, 5, N, K)
    bias = rng.integers(-200, 200, N).astype(np.int32)
    C8 = np.zeros((M, N), np.int8)
    run("gemm_tile_bias_relu_i8", (ptr(A), ptr(B), ptr(bias), ptr(C8), M, N, K), A=A, B=B, bias=bias,
        out=C8)
    lut = s8(-128, 128, 256)
    a["gelu_lut"] = lut
    M, N, K = 50, 60, 64
    A, B = s8(-4, 5, M, K), s8(-4, 5, K, N)
    bias = rng.integers(-150, 150, N).astype(np.int32)
    o = np.zeros((M, N), np.int8)
    run("gemm_bias_gelu", (ptr(A), ptr(B), ptr(bias), ptr(lut), ptr(o), M, N, K), A=A, B=B,
        bias=bias, out=o)
    o = np.zeros((M, N), np.int8)
    run("i8_gemm_gelu_lut", (ptr(A), ptr(B), ptr(lut), ptr(o), M, N, K), out=o)
    M, N, K = 32, 48, 40
    A, Bt = s8(-4, 5, M, K), s8(-4, 5, N, K)
    bias = rng.integers(-150, 150, N).astype(np.int32)
    o = np.zeros((M, N), np.int8)
    run("ffn_up_gelu_i8", (ptr(A), ptr(Bt), ptr(bias), ptr(lut), ptr(o), M, N, K), A=A, B=Bt,
        bias=bias, out=o)
    M, N, K = 60, 70, 90
    A, B, res = s8(-128, 128, M, K), s8(-128, 128, K, N), s8(-128, 128, M, N)
    o = np.zeros((M, N), np.int8)
    run("matmul_residual_add_i8", (ptr(A), ptr(B), ptr(res), ptr(o), M, N, K, C.c_int32(1 << 30), 42),
        A=A, B=B, res=res, out=o)
    M, K, V, D = 8, 16, 32, 16
    A, W1, W2 = s8(-128, 128, M, K), s8(-128, 128, K, V), s8(-128, 128, V, D)
    b1 = rng.integers(-20000, 20000, V).astype(np.int32)
    b2 = rng.integers(-2000, 2000, D).astype(np.int32)
    o = np.zeros((M, D), np.int8)
    run("ffn_relu_block", (ptr(A), ptr(W1), ptr(b1), ptr(W2), ptr(b2), ptr(o), M, K, V, D,
                           C.c_int32(1 << 24), 30, C.c_int8(-3)),
        A=A, W1=W1, b1=b1, W2=W2, b2=b2, out=o)
    save("i8_acc_callers", **a)


def gen_dot_callers(ref):
    # The matrix-vector, dot-product, narrow-GEMM, outer-product, FFN-down,
    # table-activation MLP and SiLU-gate bundles through their reference.c:
    # full-range operands where the reference's int32 sums stay defined
    # (i8_dot_i32_dma also in its harness's [-16, 16] range;
    # i16_dot_i32_dma accumulates in int64 and keeps the low 32 bits, so its
    # full-range case wraps); small-range operands where a table must be hit
    # inside its range; mlp_block at its reference's fixed hidden buffer
    # (M * V <= 256).
    rng = np.random.default_rng(131)
    s8 = lambda lo, hi, *sh: rng.integers(lo, hi, sh, dtype=np.int8)
    a = {}

    def run(name, args, **arrs):
        getattr(ref, "ref_" + name)(*args)
        for k, v in arrs.items():
            a[f"{name}__{k}"] = v

    for t, (M, K) in enumerate(((256, 130), (300, 1000))):
        A, x = s8(-128, 128, M, K), s8(-128, 128, K)
        y = np.zeros(M, np.int32)
        run("i8_matvec", (ptr(A), ptr(x), ptr(y), M, K), **{f"A{t}": A, f"x{t}": x, f"out{t}": y})
    M, N, K = 70, 90, 110
    A, Bt = s8(-128, 128, M, K), s8(-128, 128, N, K)
    bias = rng.integers(-2**20, 2**20, N).astype(np.int32)
    for t, (mult, shift) in enumerate(((1 << 10, 25), (-7, 17), (3, 0))):
        o = np.zeros((M, N), np.int8)
        run("ffn_down_i8", (ptr(A), ptr(Bt), ptr(bias), ptr(o), M, N, K, C.c_int32(mult), shift),
            **{f"out{t}": o})
    a.update(ffn_down_i8__A=A, ffn_down_i8__B=Bt, ffn_down_i8__bias=bias)
    for t, (n, lo, hi) in enumerate(((65549, -16, 17), (100003, -128, 128))):
        x, y = s8(lo, hi, n), s8(lo, hi, n)
        o = np.zeros(1, np.int32)
        run("i8_dot_i32_dma", (ptr(x), ptr(y), n, ptr(o)), **{f"a{t}": x, f"b{t}": y, f"out{t}": o})
    for t, n in enumerate((65543, 1000)):
        x = rng.integers(-32768, 32768, n).astype(np.int16)
        y = rng.integers(-32768, 32768, n).astype(np.int16)
        o = np.zeros(1, np.int32)
        run("i16_dot_i32_dma", (ptr(x), ptr(y), n, ptr(o)), **{f"a{t}": x, f"b{t}": y, f"out{t}": o})
    for t, g in enumerate((261, 1000)):
        x, y = s8(-128, 128, 4 * g), s8(-128, 128, 4 * g)
        o = np.zeros(g, np.int32)
        run("hvx_vrmpy_i8_dot", (ptr(x), ptr(y), ptr(o), g), **{f"a{t}": x, f"b{t}": y, f"out{t}": o})
    M, K, N = 161, 8101, 4
    A, X = s8(-128, 128, M, K), s8(-128, 128, K, N)
    o = np.zeros((M, N), np.int32)
    run("vtcm_stage_matmul_i8", (ptr(A), ptr(X), ptr(o), M, K, N), A=A, X=X, out=o)
    for t, (M, N) in enumerate(((128, 128), (33, 200))):
        x, y = s8(-128, 128, M), s8(-128, 128, N)
        o = np.zeros((M, N), np.int32)
        run("i8_outer_product", (ptr(x), ptr(y), ptr(o), M, N), **{f"a{t}": x, f"b{t}": y, f"out{t}": o})
    M, K, V, D = 8, 16, 32, 16
    A, W1, W2 = s8(-4, 5, M, K), s8(-4, 5, K, V), s8(-8, 9, V, D)
    b1 = rng.integers(-150, 150, V).astype(np.int32)
    b2 = rng.integers(-2000, 2000, D).astype(np.int32)
    lut = s8(-128, 128, 256)
    a.update(mlp_block__A=A, mlp_block__W1=W1, mlp_block__W2=W2, mlp_block__b1=b1, mlp_block__b2=b2,
             mlp_block__lut=lut)
    for t, (mult, shift, zp) in enumerate(((3, 10, 0), (7, 11, -3))):
        o = np.zeros((M, D), np.int8)
        run("mlp_block", (ptr(A), ptr(W1), ptr(b1), ptr(lut), ptr(W2), ptr(b2), ptr(o), M, K, V, D,
                          C.c_int32(mult), shift, C.c_int8(zp)), **{f"out{t}": o})
    silu = s8(-128, 128, 256)
    a["mlp_gate_silu_i8__lut"] = silu
    for t, (n, mult, shift) in enumerate(((150, 3, 7), (150, 5, 3), (100003, 1 << 20, 27))):
        gate, up = s8(-128, 128, n), s8(-128, 128, n)
        o = np.zeros(n, np.int8)
        run("mlp_gate_silu_i8", (ptr(gate), ptr(up), ptr(silu), ptr(o), n, C.c_int32(mult), shift),
            **{f"gate{t}": gate, f"up{t}": up, f"out{t}": o})
    save("dot_callers", **a)


def gen_sparse_attn(ref):
    # i8_sparse_attn_block through its reference.c (fixed H 1, SEQ 8,
    # HEAD_DIM 16): full-range Q / K / V, random exp tables, the band widths
    # 0 (diagonal only), 1, 2 and 7 (no key masked) and two requant sets.
    rng = np.random.default_rng(137)
    a = {}
    t = 0
    for window in (0, 1, 2, 7):
        for smult, sshift, amult, ashift in ((3, 7, 5, 8), (1 << 12, 17, 77, 14)):
            Q, K, V = (rng.integers(-128, 128, (1, 8, 16), dtype=np.int8) for _ in range(3))
            lut = rng.integers(0, 256, 256, dtype=np.uint8)
            lut[255] = 255
            o = np.zeros((1, 8, 16), np.int8)
            ref.ref_i8_sparse_attn_block(ptr(Q), ptr(K), ptr(V), ptr(lut), ptr(o), window,
                                         C.c_int32(smult), sshift, C.c_int32(amult), ashift)
            a.update({f"Q{t}": Q, f"K{t}": K, f"V{t}": V, f"lut{t}": lut, f"out{t}": o,
                      f"params{t}": np.array([window, smult, sshift, amult, ashift], np.int64)})
            t += 1
    save("sparse_attn", **a)


def gen_cache_rope(ref):
    # kv_cache_update and rope_pair_fp16 through their reference.c: caches at
    # the harness's shape (positions 0 and 63) and a ragged one (head_dim
    # 20); rotations of N(0, 4) fp16 pairs by random angles at the harness's
    # n (100) and a longer odd n.
    rng = np.random.default_rng(139)
    a = {}
    for t, (heads, cl, hd, pos) in enumerate(((4, 64, 32, 0), (4, 64, 32, 63), (3, 50, 20, 17))):
        kc, vc = (rng.integers(-128, 128, (heads, cl, hd), dtype=np.int8) for _ in range(2))
        kn, vn = (rng.integers(-128, 128, (heads, hd), dtype=np.int8) for _ in range(2))
        a.update({f"kc{t}": kc.copy(), f"vc{t}": vc.copy(), f"kn{t}": kn, f"vn{t}": vn,
                  f"pos{t}": np.array(pos)})
        ref.ref_kv_cache_update(ptr(kc), ptr(vc), ptr(kn), ptr(vn), pos, heads, cl, hd)
        a.update({f"kout{t}": kc, f"vout{t}": vc})
    for t, n in enumerate((100, 4099)):
        x = (rng.standard_normal(2 * n) * 4).astype(np.float16)
        th = rng.uniform(-np.pi, np.pi, n)
        c, sn = np.cos(th).astype(np.float16), np.sin(th).astype(np.float16)
        o = np.zeros(2 * n, np.float16)
        ref.ref_rope_pair_fp16(ptr(x), ptr(c), ptr(sn), ptr(o), n)
        a.update({f"x{t}": x, f"cos{t}": c, f"sin{t}": sn, f"rope{t}": o})
    save("cache_rope", **a)


def gen_blocks(ref):
    # i8_ffn_block, i8_ffn_swiglu_block and i8_transformer_encoder_block
    # through their reference.c: the harnesses' shapes and value ranges (X in
    # 0..3, small weights, +-4000 bias columns that kill / saturate) and
    # full-range operands at ragged shapes, where the 12-bit fields wrap;
    # within each reference's fixed scratch arrays (S * Dff <= 65536; the
    # encoder's S, D <= 64, Dff <= 128).
    rng = np.random.default_rng(149)
    a = {}

    def ints(lo, hi, *sh, dt=np.int8):
        return rng.integers(lo, hi, sh).astype(dt)

    for t, (S, D, F, small) in enumerate(((64, 128, 128, True), (37, 72, 100, False))):
        X = ints(0, 4 if small else 256, S, D, dt=np.uint8)
        W1, W2 = (ints(-3, 4, D, F), ints(-2, 3, F, D)) if small else (ints(-128, 128, D, F), ints(-128, 128, F, D))
        b1, b2 = ints(-64, 65, F, dt=np.int32), ints(-256, 257, D, dt=np.int32)
        b1[:2], b2[:2] = (-4000, 4000), (-4000, 4000)
        o = np.zeros((S, D), np.int8)
        ref.ref_i8_ffn_block(ptr(X), ptr(W1), ptr(b1), ptr(W2), ptr(b2), ptr(o), S, D, F)
        a.update({f"ffn_X{t}": X, f"ffn_W1{t}": W1, f"ffn_b1{t}": b1, f"ffn_W2{t}": W2, f"ffn_b2{t}": b2,
                  f"ffn_out{t}": o})
    for t, (S, D, F, small) in enumerate(((64, 64, 128, True), (50, 40, 96, False))):
        X = ints(0, 4 if small else 256, S, D, dt=np.uint8)
        if small:
            Wg, Wu, Wd = ints(-3, 4, D, F), ints(-3, 4, D, F), ints(-1, 2, F, D)
        else:
            Wg, Wu, Wd = ints(-128, 128, D, F), ints(-128, 128, D, F), ints(-128, 128, F, D)
        bd = ints(-256, 257, D, dt=np.int32)
        lut = ints(0, 256, 256, dt=np.uint8)
        o = np.zeros((S, D), np.int8)
        ref.ref_i8_ffn_swiglu_block(ptr(X), ptr(Wg), ptr(Wu), ptr(Wd), ptr(bd), ptr(lut), ptr(o), S, D, F)
        a.update({f"sw_X{t}": X, f"sw_Wg{t}": Wg, f"sw_Wu{t}": Wu, f"sw_Wd{t}": Wd, f"sw_bd{t}": bd,
                  f"sw_lut{t}": lut, f"sw_out{t}": o})
    for t, (S, D, F, small) in enumerate(((64, 64, 128, True), (40, 48, 100, False))):
        X = ints(0, 4 if small else 256, S, D, dt=np.uint8)
        W1, W2 = (ints(-3, 4, D, F), ints(-2, 3, F, D)) if small else (ints(-128, 128, D, F), ints(-128, 128, F, D))
        b1, b2 = ints(-64, 65, F, dt=np.int32), ints(-256, 257, D, dt=np.int32)
        b1[:2], b2[:2] = (-4000, 4000), (-4000, 4000)
        lut = np.round(255 * np.exp((np.arange(256) - 255) / 16.0)).astype(np.uint8)
        if not small:
            lut = ints(0, 256, 256, dt=np.uint8)
            lut[255] = 255
        o = np.zeros((S, D), np.int8)
        ref.ref_i8_transformer_encoder_block(ptr(X), ptr(W1), ptr(b1), ptr(W2), ptr(b2), ptr(lut), ptr(o),
                                             S, D, F)
        a.update({f"enc_X{t}": X, f"enc_W1{t}": W1, f"enc_b1{t}": b1, f"enc_W2{t}": W2, f"enc_b2{t}": b2,
                  f"enc_lut{t}": lut, f"enc_out{t}": o})
    save("blocks", **a)


def gen_affine(ref):
    # The integer affine requant bundles and the uint8 extremes through their
    # reference.c: full-range inputs (int16, int8, int32 accumulators within
    # the range where the reference's int32 products stay defined) at a
    # length off every vector width, each bundle's runtime parameters swept.
    rng = np.random.default_rng(151)
    a = {}
    n = 4099

    def run(name, t, args, **arrs):
        getattr(ref, "ref_" + name)(*args)
        for k, v in arrs.items():
            a[f"{name}__{k}{t}"] = v

    x16 = rng.integers(-32768, 32768, n).astype(np.int16)
    o = np.zeros(n, np.int8)
    run("rescale_i16_i8_dma", 0, (ptr(x16), ptr(o), n), a=x16, out=o)
    x8 = rng.integers(-128, 128, n).astype(np.int8)
    a["x8"] = x8
    for t, (zp, scale, shift) in enumerate(((0, 1, 0), (-7, 300, 3), (100, -77777, 11), (-128, 2**22, 31))):
        o = np.zeros(n, np.int16)
        run("dequant_i8_i16_dma", t, (ptr(x8), ptr(o), n, C.c_int8(zp), C.c_int32(scale), shift), out=o)
    acc = rng.integers(-(2**26), 2**26, n).astype(np.int32)
    acc[:4] = (0, -1, 7, -8)
    o = np.zeros(n, np.int8)
    run("hmx_requant_store_i8", 0, (ptr(acc), ptr(o), n), a=acc, out=o)
    for t, bias in enumerate((0, 77, -200, 100000)):
        o = np.zeros(n, np.int8)
        run("i8_add_bias_sat_dma", t, (ptr(x8), ptr(o), n, C.c_int32(bias)), out=o)
    for t, (scale, sh, s) in enumerate(((1, 0, 0), (3, 5, 2), (-1000, 333, 9), (2**31 - 1, -(2**31), 40))):
        o = np.zeros(n, np.int8)
        run("i8_element_affine_dma", t, (ptr(x8), ptr(o), n, C.c_int32(scale), C.c_int32(sh), s), out=o)
    u8 = rng.integers(0, 256, n).astype(np.uint8)
    a["u8"] = u8
    for name in ("u8_max_dma", "u8_min_dma"):
        for t, m in enumerate((n, 1, 0)):
            o = np.zeros(1, np.uint8)
            run(name, t, (ptr(u8), m, ptr(o)), out=o)
    for name in ("i8_relu_dma", "i8_relu_stream_dma"):
        o = np.zeros(n, np.int8)
        run(name, 0, (ptr(x8), ptr(o), n), out=o)
    for t, scale in enumerate((10, 0, 21, 22, 100, -3)):
        o = np.zeros(n, np.int8)
        run("i8_relu6_dma", t, (ptr(x8), ptr(o), n, C.c_int8(scale)), out=o)
    for name in ("u8_clamp_range_dma", "dma_double_buffer_relu_u8"):
        o = np.zeros(n, np.uint8)
        run(name, 0, (ptr(u8), ptr(o), n), out=o)
    for t, m in enumerate((n, 1, 77)):
        for name, src, dt in (("i8_global_avgpool_dma", x8, np.int8), ("u8_global_avgpool_dma", u8, np.uint8),
                              ("i8_global_maxpool_dma", x8, np.int8)):
            o = np.zeros(1, dt)
            run(name, t, (ptr(src), m, ptr(o)), out=o)
    o = np.zeros(1, np.int8)
    run("i8_global_maxpool_dma", 3, (ptr(x8), 0, ptr(o)), out=o)
    o = np.zeros(n, np.uint8)
    run("u8_threshold_dma", 0, (ptr(u8), ptr(o), n), out=o)
    o = np.zeros(n, np.int8)
    run("i8_sign_dma", 0, (ptr(x8), ptr(o), n), out=o)
    for t, (M, N, K) in enumerate(((32, 32, 66), (70, 90, 130))):
        A16 = rng.integers(-32768, 32768, (M, K)).astype(np.int16)
        B16 = rng.integers(-32768, 32768, (K, N)).astype(np.int16)
        o = np.zeros((M, N), np.int32)
        run("i16_gemm", t, (ptr(A16), ptr(B16), ptr(o), M, N, K), A=A16, B=B16, out=o)
    y8 = rng.integers(-128, 128, n).astype(np.int8)
    a["y8"] = y8
    for name in ("i8_add_dma", "i8_add_stream_dma", "i8_vadd_dma"):
        o = np.zeros(n, np.int8)
        run(name, 0, (ptr(x8), ptr(y8), ptr(o), n), out=o)
    save("affine", **a)


def gen_mixers(ref):
    # i8_channel_mix_block and i8_token_mix_block (fixed 8 x 16, hidden 16)
    # and rnn_cell_i8 through their reference.c: full-range int8 operands,
    # biases around the accumulator scale, the harnesses' requant sets and a
    # wider one; the RNN at H = I = 32 and a ragged H 40, I 24.
    rng = np.random.default_rng(157)
    s8 = lambda *sh: rng.integers(-128, 128, sh).astype(np.int8)
    i32 = lambda lim, *sh: rng.integers(-lim, lim, sh).astype(np.int32)
    a = {"lut": s8(256)}
    X, W1, W2 = s8(8, 16), s8(16, 16), s8(16, 16)
    b1, b2 = i32(20000, 16), i32(20000, 16)
    a.update(X=X, W1=W1, W2=W2, b1=b1, b2=b2)
    for t, (m1, s1, m2, s2) in enumerate(((3, 7, 5, 8), (1, 4, 2, 5), (1 << 12, 20, 77, 14))):
        o = np.zeros((8, 16), np.int8)
        ref.ref_i8_channel_mix_block(ptr(X), ptr(W1), ptr(b1), ptr(W2), ptr(b2), ptr(a["lut"]), ptr(o),
                                     C.c_int32(m1), s1, C.c_int32(m2), s2)
        a[f"cmix{t}"] = o
        o = np.zeros((8, 16), np.int8)
        Wt, Wt2, bt2 = W1[:, :8].copy(), W2[:8, :].copy(), b2[:8].copy()
        ref.ref_i8_token_mix_block(ptr(X), ptr(Wt), ptr(b1), ptr(Wt2), ptr(bt2), ptr(o),
                                   C.c_int32(m1), s1, C.c_int32(m2), s2)
        a.update({f"tmix{t}": o, "Wt": Wt, "Wt2": Wt2, "bt2": bt2})
    for t, (H, I, mult, shift, zp) in enumerate(((32, 32, 3, 7, 0), (32, 32, 5, 5, -3),
                                                  (40, 24, 1 << 14, 22, 9))):
        Wx, Wh, x, h = s8(H, I), s8(H, H), s8(I), s8(H)
        b = i32(30000, H)
        o = np.zeros(H, np.int8)
        ref.ref_rnn_cell_i8(ptr(Wx), ptr(Wh), ptr(b), ptr(x), ptr(h), ptr(o), H, I, C.c_int32(mult), shift,
                            C.c_int8(zp), ptr(a["lut"]))
        a.update({f"rnn_Wx{t}": Wx, f"rnn_Wh{t}": Wh, f"rnn_b{t}": b, f"rnn_x{t}": x, f"rnn_h{t}": h,
                  f"rnn_out{t}": o, f"rnn_p{t}": np.array([mult, shift, zp])})
    save("mixers", **a)


def gen_int_rows(ref):
    # The attention-tile callers, the integer layernorms with an inverse-
    # variance table, the exp-table softmax tiles, the int16 requant, the
    # per-channel double requant and the GELU FFN block through their
    # reference.c: full-range int8 operands; int16 layernorms with |gamma| <=
    # 1024 (the reference's int32 products stay defined); the fixed shapes of
    # the tile and FFN references.
    rng = np.random.default_rng(113)
    s8 = lambda *sh: rng.integers(-128, 128, sh, dtype=np.int8)
    u8 = lambda *sh: rng.integers(0, 256, sh, dtype=np.uint8)
    a = {}

    def run(name, args, **arrs):
        getattr(ref, "ref_" + name)(*args)
        for k, v in arrs.items():
            a[f"{name}__{k}"] = v

    M, N, D = 40, 50, 64
    for name, kshape in (("attention_qkt_tile", (N, D)), ("qkt_tile_i8", (D, N))):
        Q, K = s8(M, D), s8(*kshape)
        S = np.zeros((M, N), np.int8)
        run(name, (ptr(Q), ptr(K), ptr(S), M, N, D, C.c_int32(1 << 20), 26), Q=Q, K=K, out=S)
    for name, vshape in (("attention_av_tile", (N, D)), ("av_tile_i8", (D, N))):
        A, V = s8(M, N), s8(*vshape)
        O = np.zeros((M, D), np.int32)
        run(name, (ptr(A), ptr(V), ptr(O), M, N, D), A=A, V=V, out=O)
    raw = rng.integers(-2**31, 2**31, (33, 47), dtype=np.int64).astype(np.int32)
    o16 = np.zeros((33, 47), np.int16)
    run("attention_scale_i16", (ptr(raw), ptr(o16), 33, 47, C.c_int32(1 << 20), 30), raw=raw, out=o16)
    lut_e = u8(511)
    lut_e[255] = max(int(lut_e[255]), 1)
    a["exp_lut"] = lut_e
    A, B = s8(16, 16), s8(16, 16)
    o = np.zeros((16, 16), np.uint8)
    run("i8_gemm_softmax_tile", (ptr(A), ptr(B), ptr(o), ptr(lut_e)), A=A, B=B, out=o)
    Q, K = s8(16, 32), s8(16, 32)
    o = np.zeros((16, 16), np.uint8)
    run("matmul_softmax_tile", (ptr(Q), ptr(K), ptr(o), ptr(lut_e), C.c_int32(3000), 12), Q=Q, K=K, out=o)
    inv = u8(256)
    a["inv_lut"] = inv
    R, W = 37, 200
    x, g, b = s8(R, W), s8(W), s8(W)
    o = np.zeros((R, W), np.int8)
    run("i8_layernorm_dma", (ptr(x), ptr(o), R, W, ptr(g), ptr(b), ptr(inv)), x=x, gamma=g, beta=b, out=o)
    H, Wd, Cc = 9, 11, 5
    x, g, b, cl = s8(Cc, H * Wd), s8(Cc), s8(Cc), u8(Cc, 256)
    o = np.zeros((Cc, H * Wd), np.int8)
    run("i8_instance_norm", (ptr(x), ptr(o), H, Wd, Cc, ptr(g), ptr(b), ptr(cl)), x=x, gamma=g, beta=b,
        lut=cl, out=o)
    n, G = 7 * 60 + 3, 7
    x, g, b = s8(n), s8(n), s8(n)
    o = np.zeros(n, np.int8)
    run("i8_chunk_norm", (ptr(x), ptr(o), n, G, ptr(g), ptr(b), ptr(inv)), x=x, gamma=g, beta=b, out=o)
    n = 256
    x, r, g, b = s8(n), s8(n), s8(n), s8(n)
    o = np.zeros(n, np.int8)
    run("layernorm_residual", (ptr(x), ptr(r), ptr(o), n, ptr(g), ptr(b), ptr(inv)), x=x, res=r, gamma=g,
        beta=b, out=o)
    tab, idx = s8(50, 64), rng.integers(0, 50, 40).astype(np.int32)
    g, b = s8(64), s8(64)
    o = np.zeros((40, 64), np.int8)
    run("embedding_layer_norm", (ptr(tab), ptr(idx), ptr(o), 40, 64, ptr(g), ptr(b), ptr(inv)), table=tab,
        idx=idx, gamma=g, beta=b, out=o)
    R, Cc = 9, 300
    inv16 = rng.integers(0, 65536, 256).astype(np.uint16)
    a["inv_lut16"] = inv16
    x = rng.integers(-32768, 32768, (R, Cc)).astype(np.int16)
    for name, gn in (("layernorm_row_i16", Cc), ("layernorm_affine_i16", R)):
        g = rng.integers(-1024, 1025, gn).astype(np.int16)
        b = rng.integers(-32768, 32768, gn).astype(np.int16)
        o = np.zeros((R, Cc), np.int16)
        run(name, (ptr(x), ptr(o), R, Cc, ptr(g), ptr(b), ptr(inv16)), x=x, gamma=g, beta=b, out=o)
    n = 16 * 130 + 5
    x = s8(n)
    o = np.zeros(n, np.int8)
    run("i8_norm_requant_dma", (ptr(x), ptr(o), n), x=x, out=o)
    M, K, V, D = 8, 16, 32, 16
    x, W1, W2, xr = s8(M, K), s8(K, V), s8(V, D), s8(M, D)
    b1 = rng.integers(-3000, 3000, V).astype(np.int32)
    b2 = rng.integers(-3000, 3000, D).astype(np.int32)
    gl, g, b = s8(256), s8(D), s8(D)
    o = np.zeros((M, D), np.int8)
    run("gelu_ffn_residual", (ptr(x), ptr(W1), ptr(b1), ptr(gl), ptr(W2), ptr(b2), ptr(xr), ptr(g), ptr(b),
                              ptr(inv), ptr(o), M, K, V, D),
        x=x, W1=W1, b1=b1, gelu_lut=gl, W2=W2, b2=b2, x_res=xr, gamma=g, beta=b, out=o)
    save("int_rows", **a)


def gen_softmax_rms(ref):
    # The exp-table row softmaxes (division, reciprocal table, int16) and the
    # RMS norms (int8 residual + table, fp16 per-row gain, fp16 per-column
    # gamma) through their reference.c at ragged shapes; int16 softmax rows
    # of <= 8000 values so the reference's int32 sum stays defined.
    rng = np.random.default_rng(127)
    a = {}

    def run(name, args, **arrs):
        getattr(ref, "ref_" + name)(*args)
        for k, v in arrs.items():
            a[f"{name}__{k}"] = v

    R, Cc = 37, 301
    x = rng.integers(-128, 128, (R, Cc), dtype=np.int8)
    lut = rng.integers(0, 256, 256, dtype=np.uint8)
    lut[255] |= 1
    rl = rng.integers(0, 65536, 256, dtype=np.uint16)
    a.update(exp_lut=lut, recip_lut=rl, x8=x)
    o = np.zeros((R, Cc), np.uint8)
    run("softmax_rowwise", (ptr(x), ptr(o), R, Cc, ptr(lut)), out=o)
    o = np.zeros((R, Cc), np.uint8)
    run("softmax_row_i8", (ptr(x), ptr(o), R, Cc, ptr(lut), ptr(rl)), out=o)
    x16 = rng.integers(-3000, 3000, (9, 4000)).astype(np.int16)
    l16 = rng.integers(0, 65536, 256).astype(np.uint16)
    l16[255] |= 1
    o = np.zeros_like(x16)
    run("softmax_row_lut_i16", (ptr(x16), ptr(o), 9, 4000, ptr(l16)), x=x16, lut=l16, out=o)
    n = 256
    xi, ri, g = (rng.integers(-128, 128, n, dtype=np.int8) for _ in range(3))
    inv = rng.integers(0, 256, 256, dtype=np.uint8)
    o = np.zeros(n, np.int8)
    run("rmsnorm_residual", (ptr(xi), ptr(ri), ptr(o), n, ptr(g), ptr(inv)), x=xi, res=ri, gamma=g, inv=inv,
        out=o)
    xf = rng.standard_normal((33, 520)).astype(np.float16)
    gain = rng.standard_normal(33).astype(np.float16)
    o = np.zeros_like(xf)
    run("rmsnorm_gain_fp16", (ptr(xf), ptr(gain), ptr(o), 33, 520), x=xf, gain=gain, out=o)
    gam = rng.standard_normal(520).astype(np.float16)
    o = np.zeros_like(xf)
    run("rmsnorm_row_fp16", (ptr(xf), ptr(gam), ptr(o), 33, 520), gamma=gam, out=o)
    save("softmax_rms", **a)


def main():
    if not (REF_ROOT / "kernels").is_dir():
        sys.exit(f"reference tree not found at {REF_ROOT}")
    ref = load_ref()
    if len(sys.argv) > 1:                       # named generators only
        for name in sys.argv[1:]:
            fn = globals()[name]
            fn() if name == "gen_mined_fp32_sum" else fn(ref)
        return
    gen_i8_gemm_requant(ref)
    gen_i8_gemm_requant_256(ref)
    gen_i8_gemm_bias_requant(ref)
    gen_gemm_tile_zp_i8(ref)
    gen_requant_per_channel(ref)
    gen_requantize_i32_u8(ref)
    gen_gemm_u8s8_pc(ref)
    gen_hmx(ref)
    gen_hmx_family(ref)
    gen_requant_family(ref)
    gen_int8_attention_hmx(ref)
    gen_int8_attention_blocks(ref)
    gen_f16_family(ref)
    gen_i8_callers(ref)
    gen_reduce_family(ref)
    gen_i8_acc_callers(ref)
    gen_int_rows(ref)
    gen_softmax_rms(ref)
    gen_dot_callers(ref)
    gen_sparse_attn(ref)
    gen_cache_rope(ref)
    gen_blocks(ref)
    gen_affine(ref)
    gen_mixers(ref)
    gen_f16_gemms(ref)
    gen_flash_attention(ref)
    gen_online_softmax_step(ref)
    gen_rows(ref)
    gen_mined_fp32_sum()


if __name__ == "__main__":
    main()
