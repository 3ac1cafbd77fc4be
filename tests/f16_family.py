"""The fp16 post-op GEMM bundles: per bundle the golden arrays' roles and the
gemm_f16_ex arguments that compute it (kernels/expert/<bundle>/reference.c).
Used by the CPU and GPU tests."""
import numpy as np

ACT = {"none": 0, "relu": 1, "leaky": 2, "gelu": 3, "sigmoid": 4, "tanh": 5}

# bundle -> (A key, B key, b_transposed, extra kwargs)
F16_BUNDLES = {
    "fp16_matmul_gelu_hmx": ("A", "B", False, dict(act="gelu", preround=True)),
    "fp16_matmul_hmx_32x32": ("A", "B", False, dict()),
    "hmx_matmul_fp16_32": ("A", "B", False, dict()),
    "hmx_matmul_fp16_relu": ("A", "B", False, dict(act="relu")),
    "hmx_conv1x1_fp16": ("A", "B", True, dict()),
    "fp16_matmul_hmx_deepk": ("A", "B", False, dict()),
    "fp16_matmul_leaky_relu_hmx": ("A", "B", False, dict(act="leaky", preround=True)),
    "hmx_matmul_fp16_bias": ("A", "B", False, dict(bias="bias")),
    "hmx_tile_mac_fp16_32": ("A", "B", False, dict(res="C")),
    "qkt_tile_fp16": ("Q", "K", False, dict(preround=True, scale=0.125)),
    "av_tile_fp16": ("A", "V", True, dict()),
    # the accumulator rounded to fp16 before the adds and the activation
    "fp16_matmul_bias_gelu": ("A", "B", False, dict(bias="bias", act="gelu", preround="acc")),
    "fp16_matmul_bias_relu": ("A", "B", False, dict(bias="bias", act="relu", preround="acc")),
    "fp16_matmul_residual": ("A", "B", False, dict(res="C", preround="acc")),
    "fp16_matmul_sigmoid": ("A", "B", False, dict(act="sigmoid", preround="acc")),
    "fp16_matmul_tanh": ("A", "B", False, dict(act="tanh", preround="acc")),
    "ai_fp16_matmul_gelu": ("A", "B", False, dict(act="gelu", preround="acc")),
}


def f16_case(g, bundle):
    """(A, B, expected, kwargs for gemm_f16_ex) of a bundle from f16_family.npz."""
    ak, bk, bt, kw = F16_BUNDLES[bundle]
    arr = {k.split("__", 1)[1]: g[k] for k in g if k.startswith(bundle + "__")}
    kw = dict(kw)
    for role in ("bias", "res"):
        if role in kw:
            kw[role] = arr[kw[role]]
    kw["b_transposed"] = bt
    return arr[ak], arr[bk], arr["out"], kw
