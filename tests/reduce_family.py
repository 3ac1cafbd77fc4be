"""The integer reduction bundles: per bundle its candidate_kernel parameters
(in order), the element type of its array operands, and the library call
that computes it (kernels/expert/<bundle>/kernel_api.h and reference.c).
Used by the golden generator and by the CPU and GPU tests.

kind:  ("reduce", op)          hexcuda_reduce_int (op of HEXCUDA_RED_*)
       ("minmax", op, scalar)  hexcuda_minmax_ew
       ("group_sum",)          hexcuda_group_sum_i8 (w = 4)
       ("scan",)               hexcuda_scan_max_i8
       ("gqa",)                hexcuda_head_group_reduce_i8
"""
import ctypes as C

import numpy as np

I8, U8, I16, I32 = np.int8, np.uint8, np.int16, np.int32

RD_BUNDLES = {
    "vtcm_reduce_i32": (("a", "n", "out"), I32, ("reduce", "sum")),
    "i8_sum_dma": (("a", "n", "out"), I8, ("reduce", "sum")),
    "dma_double_buffer_reduce_i32": (("a", "n", "out"), I32, ("reduce", "sum64")),
    "i8_sumsq_i32": (("a", "n", "out"), I8, ("reduce", "sumsq")),
    "i8_sumsq_diff_i32": (("a", "b", "n", "out"), I8, ("reduce", "sumsq_diff")),
    "i8_weighted_sum": (("a", "b", "n", "out"), I8, ("reduce", "dot")),
    "i8_l1norm_dma": (("a", "n", "out"), I8, ("reduce", "l1")),
    "i8_absmax_dma": (("a", "n", "out"), I8, ("reduce", "absmax")),
    "dma_stream_max_u8": (("a", "n", "out"), U8, ("reduce", "max")),
    "i8_argmax_dma": (("a", "n", "out"), I8, ("reduce", "argmax")),
    "i8_argmin_dma": (("a", "n", "out"), I8, ("reduce", "argmin")),
    "i8_top1_reduce_dma": (("a", "n", "out"), I8, ("reduce", "top1")),
    "i8_mean_dma": (("a", "n", "out"), I8, ("reduce", "mean")),
    "hvx_vmax_i8": (("a", "b", "out", "n"), I8, ("minmax", "max", False)),
    "hvx_vmax_u8": (("a", "b", "out", "n"), U8, ("minmax", "max", False)),
    "hvx_vmin_i16": (("a", "b", "out", "n"), I16, ("minmax", "min", False)),
    "hvx_vmin_u8": (("a", "b", "out", "n"), U8, ("minmax", "min", False)),
    "i8_max_scalar_dma": (("a", "out", "n", "c"), I8, ("minmax", "max", True)),
    "i8_min_scalar_dma": (("a", "out", "n", "c"), I8, ("minmax", "min", True)),
    "hvx_vradd_i8_reduce": (("a", "out", "g"), I8, ("group_sum",)),
    "i8_scan_max": (("a", "out", "n"), I8, ("scan",)),
    "gqa_group_reduce_i8": (("X", "Y", "H", "G", "M", "N", "mult", "shift"), I8, ("gqa",)),
}


def out_buffer(bundle, arr):
    """Zeroed output buffer of the bundle's candidate_kernel."""
    params, dt, kind = RD_BUNDLES[bundle]
    if kind[0] == "reduce":
        op = kind[1]
        if op == "sum64":
            return np.zeros(1, np.int64)
        if bundle == "dma_stream_max_u8":
            return np.zeros(1, np.uint8)
        return np.zeros(2 if op == "top1" else 1, np.int32)
    if kind[0] == "minmax":
        return np.zeros_like(arr["a"])
    if kind[0] == "group_sum":
        return np.zeros(arr["a"].size // 4, np.int32)
    if kind[0] == "scan":
        return np.zeros_like(arr["a"])
    G, M, N = (int(arr[k]) for k in ("G", "M", "N"))
    return np.zeros(G * M * N, np.int8)


def ctypes_args(bundle, arr, out):
    """candidate_kernel arguments (reference.c, shim or oracle candidate)."""
    params, dt, kind = RD_BUNDLES[bundle]
    args = []
    for prm in params:
        if prm in ("out", "Y"):
            args.append(out.ctypes.data_as(C.c_void_p))
        elif prm == "n":
            args.append(C.c_int(arr["a"].size))
        elif prm == "g":
            args.append(C.c_int(arr["a"].size // 4))
        elif prm == "c":
            args.append(C.c_int8(int(arr["c"])))
        elif prm == "mult":
            args.append(C.c_int32(int(arr["mult"])))
        elif prm in ("H", "G", "M", "N", "shift"):
            args.append(C.c_int(int(arr[prm])))
        else:
            args.append(arr[prm].ctypes.data_as(C.c_void_p))
    return args


def library_call(mod, bundle, arr):
    """The bundle's result through a module exposing reduce_int / minmax_ew /
    group_sum_i8 / scan_max_i8 / head_group_reduce_i8 (the package's ops or
    the oracle), shaped like out_buffer()."""
    params, dt, kind = RD_BUNDLES[bundle]
    if kind[0] == "reduce":
        r = mod.reduce_int(arr["a"], kind[1], arr.get("b"))
        out = out_buffer(bundle, arr)
        out[:] = r if kind[1] == "top1" else [r]
        return out
    if kind[0] == "minmax":
        if kind[2]:
            return mod.minmax_ew(arr["a"], None, int(arr["c"]), kind[1])
        return mod.minmax_ew(arr["a"], arr["b"], 0, kind[1])
    if kind[0] == "group_sum":
        return mod.group_sum_i8(arr["a"], 4)
    if kind[0] == "scan":
        return mod.scan_max_i8(arr["a"])
    H, G, M, N = (int(arr[k]) for k in ("H", "G", "M", "N"))
    return mod.head_group_reduce_i8(arr["X"].reshape(H, M * N), G, int(arr["mult"]),
                                    int(arr["shift"])).ravel()


def make_inputs(bundle, rng, n):
    """Seeded inputs of one case with n elements (n = 4 g for the group sum;
    the head-group reduce takes its own shape)."""
    params, dt, kind = RD_BUNDLES[bundle]
    info = np.iinfo(dt)
    hi = 1 << 18 if bundle == "vtcm_reduce_i32" else info.max + 1
    lo = -hi if bundle == "vtcm_reduce_i32" else info.min
    arr = {}
    if kind[0] == "gqa":
        H, G, M, N = 8, 2, 5, 33
        arr.update(X=rng.integers(-128, 128, H * M * N).astype(np.int8), H=H, G=G, M=M, N=N,
                   mult=int(rng.integers(1 << 20, 1 << 24)), shift=int(rng.integers(20, 26)))
        return arr
    arr["a"] = rng.integers(lo, hi, n, dtype=np.int64).astype(dt)
    if "b" in params:
        arr["b"] = rng.integers(lo, hi, n, dtype=np.int64).astype(dt)
    if "c" in params:
        arr["c"] = int(rng.integers(-128, 128))
    if kind[0] == "reduce" and kind[1] in ("argmax", "argmin", "top1") and n > 8:
        # ties: the extreme planted at three positions, the first one wins
        v = info.max if kind[1] != "argmin" else info.min
        for pos in sorted(rng.choice(n, 3, replace=False)):
            arr["a"][pos] = v
    return arr


def golden_cases(g):
    """(bundle, case) pairs of the reduce_family fixture."""
    return sorted({tuple(k.split("__")[:2]) for k in g})


def golden_case(g, bundle, case):
    return {k.split("__", 2)[2]: g[k] for k in g if k.startswith(f"{bundle}__{case}__")}
