"""Per-row CRC32 of the oracle's full output for the two integer GEMMs at
the benchmark shape (M=16384, N=K=8192), so that the GPU's WHOLE output can
be checked bit for bit without shipping 128-512 MB of expected output.

    python tests/golden/make_crc.py [--threads N]

writes tests/golden/crc_gemm_u8s8_pc_16384x8192x8192.npy and
tests/golden/crc_gemm_hmx_16384x8192x8192.npy (16384 uint32 each).

The inputs come from `inputs(kind)` below (numpy default_rng seeds), which the
slow GPU test calls too:
  u8s8  u8 A with zpA 128, s8 B [K, N], int32 bias round(N(0, 1000)),
        per-column mult in [2^30, 2^31), shift 44, zp_out 128 -> u8
        (the per-channel requant GEMM the benchmark times);
  hmx   u8 A, s8 B [K, N], bias U[-3000, 3000), HMX field sx12((acc*17+8)>>4)
        + bias, ReLU -> int32 (i8_matmul_bias_relu_hmx's epilogue).
The expected rows come from oracle/hexoracle.c (the restatement of the
reference's reference.c files, pinned by tests/test_oracle_golden.py), run on
all host threads; about half a minute per GEMM on 8 cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import os
import sys
import time
import zlib
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
M, N, K = 16384, 8192, 8192
FILES = {"u8s8": HERE / f"crc_gemm_u8s8_pc_{M}x{N}x{K}.npy",
         "hmx": HERE / f"crc_gemm_hmx_{M}x{N}x{K}.npy"}


def inputs(kind: str) -> dict:
    rng = np.random.default_rng({"u8s8": 20240, "hmx": 20241}[kind])
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    if kind == "u8s8":
        bias = np.round(rng.normal(0, 1000, N)).astype(np.int32)
        mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
        shift = np.full(N, 44, np.int32)
        return dict(A=A, B=B, bias=bias, mult=mult, shift=shift, zpA=128, zp_out=128)
    bias = rng.integers(-3000, 3000, N).astype(np.int32)
    return dict(A=A, B=B, bias=bias)


def row_crcs(out: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(out)
    return np.array([zlib.crc32(out[i].tobytes()) for i in range(out.shape[0])], np.uint32)


def oracle_rows(kind: str, d: dict, r0: int, r1: int) -> np.ndarray:
    from oracle import oracle as o
    lib = o.lib()
    A = np.ascontiguousarray(d["A"][r0:r1])
    n = r1 - r0
    if kind == "u8s8":
        out = np.empty((n, N), np.uint8)
        lib.oracle_gemm_u8s8_pc_rows(o._p(A), o._p(d["B"]), o._p(d["bias"]), o._p(out), n, N, K,
                                     C.c_int32(d["zpA"]), o._p(d["mult"]), o._p(d["shift"]),
                                     C.c_uint8(d["zp_out"]), 0, n)
        return out
    out = np.empty((n, N), np.int32)
    lib.oracle_gemm_hmx_ex_rows(o._p(A), o._p(d["B"]), 0, o._p(out), n, N, K, C.c_int32(0), 0, 1,
                                o._p(d["bias"]), 0, None, None, 0, 0, n)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=len(os.sched_getaffinity(0)))
    ap.add_argument("--kinds", default="u8s8,hmx")
    args = ap.parse_args()
    sys.path.insert(0, str(REPO))
    for kind in args.kinds.split(","):
        t0 = time.time()
        d = inputs(kind)
        crcs = np.zeros(M, np.uint32)
        blk = 64

        def work(r0):
            r1 = min(M, r0 + blk)
            crcs[r0:r1] = row_crcs(oracle_rows(kind, d, r0, r1))

        with ThreadPoolExecutor(args.threads) as ex:
            list(ex.map(work, range(0, M, blk)))
        np.save(FILES[kind], crcs)
        print(f"{kind}: {FILES[kind].name} in {time.time() - t0:.1f} s")


if __name__ == "__main__":
    main()
