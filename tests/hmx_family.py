"""The HMX-convention bundles that share the u8 x s8 GEMM and differ in the
post-op: per bundle its candidate_kernel parameters (in order) and the
gemm_hmx_ex arguments that compute it (kernels/expert/<bundle>/reference.c).
Used by the golden generator and by the CPU and GPU tests."""

# param kinds: A u8 [M,K]; B s8 [K,N] (Bt: [N,K]); bias i32 [N]; res32 i32 [M,N];
# res8 i8 [M,N]; lut32 i32 [256]; lut8 i8 [256]; out; n / M / N / K ints
SQ = ("A", "B", "out", "n")
BUNDLES = {
    "hmx_matmul_i8_32": (SQ, dict(store="i32")),
    "hmx_matmul_i8_accum_chain": (("A", "B", "out", "n", "K"), dict(store="i32")),
    "hmx_matmul_i8_bias": (("A", "B", "bias", "out", "n"), dict(store="i32")),
    "hmx_matmul_i8_bias_relu": (("A", "B", "bias", "out", "n"), dict(store="i32", act="relu")),
    "hmx_matmul_i8_col_major": (SQ, dict(store="i32", col_major=True)),
    "hmx_matmul_i8_gelu_lut": (("A", "B", "lut32", "out", "n"), dict(store="lut_i32")),
    "hmx_matmul_i8_multi_n": (("A", "B", "out", "M", "N", "K"), dict(store="i32")),
    "hmx_matmul_i8_rect_32x64": (("A", "B", "out", "M", "N", "K"), dict(store="i32")),
    "hmx_matmul_i8_relu": (SQ, dict(store="i32", act="relu")),
    "i8_matmul_bias_hmx": (("A", "B", "bias", "out", "n"), dict(store="i32")),
    "i8_matmul_bias_relu_hmx": (("A", "B", "bias", "out", "n"), dict(store="i32", act="relu")),
    "i8_matmul_hmx_64x64": (SQ, dict(store="u16_field")),
    "i8_matmul_hmx_96x96": (SQ, dict(store="u16_field")),
    "i8_matmul_hmx_requant": (SQ, dict(store="i8_low")),
    "i8_matmul_leaky_relu_hmx": (SQ, dict(store="i32", act="leaky_shr3")),
    "i8_matmul_residual_hmx": (("A", "B", "res32", "out", "n"), dict(store="i32")),
    "i8_matmul_add_requant_hmx": (("A", "B", "res8", "out", "n"), dict(store="i8_sat")),
    "i8_matmul_bias_gelu_hmx": (("A", "B", "bias", "lut8", "out", "n"), dict(store="lut_i8")),
    "i8_gemm_relu_hmx_deepk": (("A", "B", "out", "n", "K"), dict(store="i32", act="relu")),
    "i8_linear_proj_hmx": (("A", "Bt", "bias", "out", "n"), dict(store="i8_sat", b_transposed=True)),
    "hmx_kacc_i8_2tile": (("A", "B", "out", "n", "K"), dict(store="i32")),
    "hmx_kacc_i8_4tile": (("A", "B", "out", "n", "K"), dict(store="i32")),
    "hmx_tile_mac_i8_32": (SQ, dict(store="i32")),
    "hmx_gemv_i8": (("A", "x", "out", "n"), dict(store="i32")),
}

OUT_DTYPE = {"i32": "int32", "i8_sat": "int8", "u8_sat": "uint8", "i8_low": "int8",
             "u16_field": "uint16", "lut_i32": "int32", "lut_i8": "int8"}


def shape_of(bundle):
    """(M, N, K) of the golden case."""
    params, kw = BUNDLES[bundle]
    if "lut" in kw["store"]:
        return 32, 32, 32          # keeps |v| small enough for the 256-entry table
    if bundle == "hmx_gemv_i8":
        return 150, 1, 150
    if "M" in params:
        return (60, 100, 130) if bundle.endswith("rect_32x64") else (70, 90, 150)
    if "K" in params:
        return 72, 72, 200
    return 72, 72, 72


def ex_kwargs(bundle, arrays):
    """gemm_hmx_ex keyword arguments for a bundle from its golden arrays."""
    params, kw = BUNDLES[bundle]
    kw = dict(kw)
    if "bias" in params:
        kw["bias"] = arrays["bias"]
    if "res32" in params:
        kw["res"] = arrays["res32"]
    if "res8" in params:
        kw["res"] = arrays["res8"]
    if "lut32" in params:
        kw["lut"] = arrays["lut32"]
    if "lut8" in params:
        kw["lut"] = arrays["lut8"]
    return kw


def golden_case(g, bundle):
    """(A, B, expected out, gemm_hmx_ex kwargs) of a bundle from hmx_family.npz."""
    params, kw = BUNDLES[bundle]
    arr = {k.split("__", 1)[1]: g[k] for k in g if k.startswith(bundle + "__")}
    M, N, K = (int(v) for v in arr["mnk"])
    A = arr["A"].reshape(M, K)
    if "Bt" in arr:
        B = arr["Bt"].reshape(N, K)
    elif "x" in arr:
        B = arr["x"].reshape(K, 1)
    else:
        B = arr["B"].reshape(K, N)
    for r in ("res32", "res8"):
        if r in arr:
            arr[r] = arr[r].reshape(M, N)
    out = arr["out"].reshape((N, M) if kw.get("col_major") else (M, N))
    return A, B, out, ex_kwargs(bundle, arr)
