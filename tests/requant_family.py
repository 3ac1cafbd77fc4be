"""The elementwise requant bundles: per bundle its candidate_kernel
parameters (in order), the fixed constants of its reference.c, and the
requant_ew arguments that compute it (kernels/expert/<bundle>/reference.c).
Used by the golden generator and by the CPU and GPU tests."""

# params: a32 / a8 / b32 / b8 inputs, out, n, mult, shift, zp, lo, hi, lut
RQ_BUNDLES = {
    "bias_add_requant": (("a32", "b32", "out", "n", "mult", "shift", "zp"), dict(pre="add")),
    "epilogue_requant_i32_i8": (("a32", "out", "n", "mult", "shift"), dict()),
    "requant_relu_dma": (("a32", "out", "n"), dict(mult=13, shift=3, lo1=0, lo2=0)),
    "requant_relu6_dma": (("a32", "out", "n"), dict(mult=13, shift=3, lo1=0, hi1=24, lo2=0, hi2=24)),
    "requantize_i32_i8_dma": (("a32", "out", "n", "mult", "shift", "zp"), dict()),
    "dma_stream_requant_i32_i8": (("a32", "out", "n", "mult", "shift", "zp"), dict(sign_of_a=True)),
    "add_relu_requant": (("a32", "b32", "out", "n", "mult", "shift", "zp"), dict(pre="add_relu")),
    "residual_add_requant": (("a32", "b32", "out", "n", "mult", "shift", "zp"), dict(pre="add")),
    "requant_add_dma": (("a32", "b32", "out", "n"), dict(pre="add", mult=5, shift=3)),
    "mul_add_requant_dma": (("a32", "b32", "out", "n"), dict(pre="mul_add", pre_c=50, mult=3, shift=1)),
    "i8_mul_requant_dma": (("a8", "b8", "out", "n", "mult", "shift", "zp"), dict(pre="mul_add")),
    "i8_clip_requant_dma": (("a32", "out", "n", "mult", "shift", "zp", "lo", "hi"), dict()),
    "requant_sigmoid_lut": (("a32", "out", "n", "mult", "shift", "zp", "lut"),
                            dict(lo1=0, hi1=255, lo2=0, hi2=255)),
    "requant_tanh_lut": (("a32", "out", "n", "mult", "shift", "zp", "lut"),
                         dict(lo1=0, hi1=255, lo2=0, hi2=255)),
    "i8_skip_add_relu_requant": (("a8", "b8", "out", "n", "mult", "shift", "zp"), dict(pre="add_relu")),
}


def ew_kwargs(bundle, arr):
    """requant_ew keyword arguments of a bundle's case (arr: its arrays)."""
    params, kw = RQ_BUNDLES[bundle]
    kw = dict(kw)
    for k in ("mult", "shift", "zp"):
        if k in params:
            kw[k] = int(arr[k])
    if "lo" in params:
        kw["lo2"], kw["hi2"] = int(arr["lo"]), int(arr["hi"])
    if "lut" in params:
        kw["lut"] = arr["lut"]
    for k in ("b32", "b8"):
        if k in params:
            kw["b"] = arr[k]
    return kw


def case_arrays(g, bundle, case):
    return {k.split("__", 2)[2]: g[k] for k in g if k.startswith(f"{bundle}__{case}__")}
