// int_rows.cu -- integer row operators with the corpus's table-driven
// normalisation arithmetic, one warp per row (the rows are short: tens to a
// few thousand elements), several rows per 256-thread block:
//   hexcuda_layernorm_lut_i8   int8 layernorm with an inverse-variance table
//                              (shared, per-chunk or per-channel affine;
//                              optional saturating residual, optional gather)
//   hexcuda_layernorm_lut_i16  the int16 forms (per-column or per-row affine)
//   hexcuda_lut_softmax_u8     row softmax of int8 scores by an exp table
//   hexcuda_lut_softmax_i16    the int16 form (int64 sums, 32767 scale)
//   hexcuda_requant_i16        int32 -> int16 round-half-away requant
//   hexcuda_norm_requant_i8    per-channel requant followed by a second one
// Reference semantics: kernels/expert/<bundle>/reference.c of
// i8_layernorm_dma, i8_instance_norm, i8_chunk_norm, layernorm_residual,
// embedding_layer_norm, layernorm_row_i16, layernorm_affine_i16,
// i8_gemm_softmax_tile, matmul_softmax_tile, vtcm_softmax_row_i16,
// attention_scale_i16 and i8_norm_requant_dma.  Integer division is C's
// (truncation toward zero), shifts of negative values are arithmetic (as gcc
// compiles the references), sums wrap like the references' int32
// accumulators; every result is bit-identical.
#include "ew_launch.cuh"
#include "hx_internal.h"
#include "requant.cuh"

namespace hx {
namespace {

constexpr int kRowWarps = 8;   // rows per 256-thread block

__device__ __forceinline__ int32_t warp_sum_i32(int32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int64_t warp_sum_i64(int64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_max_i32(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int sat8(int v) { return v > 127 ? 127 : (v < -128 ? -128 : v); }
__device__ __forceinline__ int sat16(int v) { return v > 32767 ? 32767 : (v < -32768 ? -32768 : v); }

// ------------------------------------------------------------ int8 layernorm
// Row r: t = x row (x + idx[r] W when gathered; sat8(x + res) with a
// residual); mu = sum / W; var = sum (t - mu)^2 / W (int32, C division);
// inv = lut[clamp(var, 0, 255)]; out = sat8((((t - mu) g + 64) >> 7) inv + 128)
// >> 8) + b).  affine: SHARED g[j], b[j]; ROWWISE g[r W + j], b[r W + j];
// PER_ROW g[r], b[r] and the table lut + 256 r.  RMS_SHARED: mu = 0, no b
// (rmsnorm_residual/reference.c: var = sum t^2 / W, out = sat8(normed)).
__global__ void __launch_bounds__(256) layernorm_lut_i8_kernel(
    const int8_t *__restrict__ x, const int32_t *__restrict__ idx, const int8_t *__restrict__ res,
    int8_t *__restrict__ out, int R, int W, const int8_t *__restrict__ gamma,
    const int8_t *__restrict__ beta, const uint8_t *__restrict__ lut, int affine) {
    const int lane = threadIdx.x & 31;
    for (int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5); r < R; r += gridDim.x * kRowWarps) {
        const int8_t *xr = x + (size_t)(idx ? idx[r] : r) * W;
        const int8_t *rr = res ? res + (size_t)r * W : nullptr;
        auto load = [&](int j) -> int {
            int t = xr[j];
            if (rr) t = sat8(t + rr[j]);
            return t;
        };
        const bool rms = affine == HEXCUDA_LN_RMS_SHARED;
        int32_t s = 0;
        if (!rms)
            for (int j = lane; j < W; j += 32) s += load(j);
        const int32_t mu = rms ? 0 : warp_sum_i32(s) / W;
        uint32_t vs = 0;
        for (int j = lane; j < W; j += 32) {
            const int32_t d = load(j) - mu;
            vs += (uint32_t)(d * d);
        }
        const int32_t var = (int32_t)(uint32_t)warp_sum_i32((int32_t)vs) / W;
        const int vi = var < 0 ? 0 : (var > 255 ? 255 : var);
        const uint8_t *tl = affine == HEXCUDA_LN_AFFINE_PER_ROW ? lut + 256 * (size_t)r : lut;
        const int32_t inv = tl[vi];
        int8_t *orow = out + (size_t)r * W;
        for (int j = lane; j < W; j += 32) {
            int32_t g, b = 0;
            if (rms) {
                g = gamma[j];
            } else if (affine == HEXCUDA_LN_AFFINE_PER_ROW) {
                g = gamma[r];
                b = beta[r];
            } else {
                const size_t gj = affine == HEXCUDA_LN_AFFINE_ROWWISE ? (size_t)r * W + j : (size_t)j;
                g = gamma[gj];
                b = beta[gj];
            }
            const int32_t d = load(j) - mu;
            const int32_t scaled = (d * g + 64) >> 7;
            const int32_t normed = (scaled * inv + 128) >> 8;
            orow[j] = (int8_t)sat8(rms ? normed : normed + b);
        }
    }
}

// ----------------------------------------------------------- int16 layernorm
// mu = (int32)(sum / C) and var = sum (x - mu)^2 / C in int64; inv =
// lut[clamp(var >> 5, 0, 255)].  order 0 (layernorm_row_i16): out =
// sat16(((((x - mu) g[c] + 32) >> 6) inv + 512) >> 10) + b[c]); order 1
// (layernorm_affine_i16): out = sat16(((((x - mu) inv + 512) >> 10) g[r] + 32)
// >> 6) + b[r]).
__global__ void __launch_bounds__(256) layernorm_lut_i16_kernel(
    const int16_t *__restrict__ x, int16_t *__restrict__ out, int R, int C,
    const int16_t *__restrict__ gamma, const int16_t *__restrict__ beta,
    const uint16_t *__restrict__ lut, int order) {
    const int lane = threadIdx.x & 31;
    for (int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5); r < R; r += gridDim.x * kRowWarps) {
        const int16_t *xr = x + (size_t)r * C;
        int64_t s = 0;
        for (int j = lane; j < C; j += 32) s += xr[j];
        const int32_t mu = (int32_t)(warp_sum_i64(s) / C);
        int64_t vs = 0;
        for (int j = lane; j < C; j += 32) {
            const int64_t d = (int64_t)xr[j] - mu;
            vs += d * d;
        }
        const int64_t var = warp_sum_i64(vs) / C;
        int32_t vi = (int32_t)(var >> 5);
        vi = vi < 0 ? 0 : (vi > 255 ? 255 : vi);
        const int32_t inv = lut[vi];
        int16_t *orow = out + (size_t)r * C;
        for (int j = lane; j < C; j += 32) {
            const int32_t d = (int32_t)xr[j] - mu;
            int32_t v;
            if (order == 0) {
                const int32_t scaled = (d * (int32_t)gamma[j] + 32) >> 6;
                v = ((scaled * inv + 512) >> 10) + beta[j];
            } else {
                const int32_t normed = (d * inv + 512) >> 10;
                v = ((normed * (int32_t)gamma[r] + 32) >> 6) + beta[r];
            }
            orow[j] = (int16_t)sat16(v);
        }
    }
}

// ------------------------------------------------------------ LUT softmaxes
// u8: m = row max; e_j = lut[max(x_j - m, -255) + 255]; S = sum e;
// p_j = (e_j 255 + S / 2) / S  (i8_gemm_softmax_tile/reference.c, step C)
// With a reciprocal table (softmax_row_i8/reference.c): recip =
// recip_lut[clamp(S >> 6, 0, 255)], p_j = clamp((e_j recip + 32768) >> 16, 0, 255).
__global__ void __launch_bounds__(256) lut_softmax_u8_kernel(const int8_t *__restrict__ x,
                                                             uint8_t *__restrict__ out, int R,
                                                             int C,
                                                             const uint8_t *__restrict__ lut,
                                                             const uint16_t *__restrict__ recip_lut) {
    const int lane = threadIdx.x & 31;
    for (int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5); r < R; r += gridDim.x * kRowWarps) {
        const int8_t *xr = x + (size_t)r * C;
        int m = -128;
        for (int j = lane; j < C; j += 32) m = max(m, (int)xr[j]);
        m = warp_max_i32(m);
        int32_t s = 0;
        for (int j = lane; j < C; j += 32) s += lut[max((int)xr[j] - m, -255) + 255];
        s = warp_sum_i32(s);
        const int32_t half = s / 2;
        const int32_t si = s >> 6;
        const int32_t recip = recip_lut ? recip_lut[si < 0 ? 0 : (si > 255 ? 255 : si)] : 0;
        uint8_t *orow = out + (size_t)r * C;
        for (int j = lane; j < C; j += 32) {
            const int32_t e = lut[max((int)xr[j] - m, -255) + 255];
            if (recip_lut) {
                const int32_t v = (e * recip + 32768) >> 16;
                orow[j] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
            } else {
                orow[j] = (uint8_t)(s > 0 ? (e * 255 + half) / s : 0);
            }
        }
    }
}

// i16: the same with int16 scores, a uint16 table, int64 sums and
// p_j = (e_j 32767 + S / 2) / S  (vtcm_softmax_row_i16/reference.c)
__global__ void __launch_bounds__(256) lut_softmax_i16_kernel(const int16_t *__restrict__ x,
                                                              int16_t *__restrict__ out, int R,
                                                              int C,
                                                              const uint16_t *__restrict__ lut) {
    const int lane = threadIdx.x & 31;
    for (int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5); r < R; r += gridDim.x * kRowWarps) {
        const int16_t *xr = x + (size_t)r * C;
        int m = -32768;
        for (int j = lane; j < C; j += 32) m = max(m, (int)xr[j]);
        m = warp_max_i32(m);
        int64_t s = 0;
        for (int j = lane; j < C; j += 32) s += lut[max((int)xr[j] - m, -255) + 255];
        s = warp_sum_i64(s);
        const int64_t half = s / 2;
        int16_t *orow = out + (size_t)r * C;
        for (int j = lane; j < C; j += 32) {
            const int64_t e = lut[max((int)xr[j] - m, -255) + 255];
            orow[j] = (int16_t)(s > 0 ? (e * 32767 + half) / s : 0);
        }
    }
}

// ------------------------------------------------------ elementwise requants
// out = sat16(round_half_away(a * mult >> shift))  (attention_scale_i16)
__global__ void __launch_bounds__(256) requant_i16_kernel(const int32_t *__restrict__ a,
                                                          int16_t *__restrict__ out, int64_t n,
                                                          int32_t mult, int shift) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t q = rq_round((int64_t)a[i] * (int64_t)mult, shift);
        out[i] = (int16_t)(q > 32767 ? 32767 : (q < -32768 ? -32768 : q));
    }
}

// channel c = i / per_ch: v = round_half_away(a * nmult[c] >> nshift[c])
// (int64, unclamped), then out = sat8(round_half_away(v * mult >> shift) +
// zp)  (i8_norm_requant_dma/reference.c:11-22)
__global__ void __launch_bounds__(256) norm_requant_i8_kernel(
    const int8_t *__restrict__ a, int8_t *__restrict__ out, int64_t n, int64_t per_ch, int nch,
    const int32_t *__restrict__ nmult, const int *__restrict__ nshift, int32_t mult, int shift,
    int zp) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t total = per_ch * nch;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total && i < n; i += stride) {
        const int c = (int)(i / per_ch);
        const int64_t v = rq_round((int64_t)a[i] * (int64_t)nmult[c], nshift[c]);
        const int64_t r = rq_round(v * (int64_t)mult, shift) + zp;
        out[i] = (int8_t)(r > 127 ? 127 : (r < -128 ? -128 : r));
    }
}

// out = sat8(round_half_away((lut[gate + 128] up) * mult >> shift))
// (mlp_gate_silu_i8/reference.c:4-17)
__global__ void __launch_bounds__(256) gate_mul_requant_i8_kernel(
    const int8_t *__restrict__ gate, const int8_t *__restrict__ up, const int8_t *__restrict__ lut,
    int8_t *__restrict__ out, int64_t n, int32_t mult, int shift) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int32_t g = lut[(int)gate[i] + 128];
        const int64_t q = rq_round((int64_t)(g * (int32_t)up[i]) * (int64_t)mult, shift);
        out[i] = (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
    }
}

int row_blocks(const Dev *d, int R) {
    const int64_t b = ((int64_t)R + kRowWarps - 1) / kRowWarps;
    const int64_t cap = (int64_t)d->sms * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_layernorm_lut_i8(int dev, const int8_t *x, const int32_t *idx,
                                      const int8_t *res, int8_t *out, int R, int W,
                                      const int8_t *gamma, const int8_t *beta,
                                      const uint8_t *inv_lut, int affine) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || W < 1 || affine < HEXCUDA_LN_AFFINE_SHARED || affine > HEXCUDA_LN_RMS_SHARED)
        return fail(HEXCUDA_ERR_ARG, "layernorm_lut_i8: R %d W %d affine %d", R, W, affine);
    if (R == 0) return HEXCUDA_OK;
    if (!x || !out || !gamma || (!beta && affine != HEXCUDA_LN_RMS_SHARED) || !inv_lut)
        return fail(HEXCUDA_ERR_ARG, "layernorm_lut_i8: null pointer");
    launch_begin(d);
    layernorm_lut_i8_kernel<<<row_blocks(d, R), 256, 0, d->stream>>>(x, idx, res, out, R, W, gamma,
                                                                     beta, inv_lut, affine);
    return launch_end(d, "layernorm_lut_i8");
}

HX_EXPORT int hexcuda_layernorm_lut_i16(int dev, const int16_t *x, int16_t *out, int R, int C,
                                       const int16_t *gamma, const int16_t *beta,
                                       const uint16_t *inv_lut, int order) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C < 1 || (order != 0 && order != 1))
        return fail(HEXCUDA_ERR_ARG, "layernorm_lut_i16: R %d C %d order %d", R, C, order);
    if (R == 0) return HEXCUDA_OK;
    if (!x || !out || !gamma || !beta || !inv_lut)
        return fail(HEXCUDA_ERR_ARG, "layernorm_lut_i16: null pointer");
    launch_begin(d);
    layernorm_lut_i16_kernel<<<row_blocks(d, R), 256, 0, d->stream>>>(x, out, R, C, gamma, beta,
                                                                      inv_lut, order);
    return launch_end(d, "layernorm_lut_i16");
}

HX_EXPORT int hexcuda_lut_softmax_u8(int dev, const int8_t *x, uint8_t *out, int R, int C,
                                    const uint8_t *exp_lut, const uint16_t *recip_lut) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C < 1) return fail(HEXCUDA_ERR_ARG, "lut_softmax_u8: R %d C %d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (!x || !out || !exp_lut) return fail(HEXCUDA_ERR_ARG, "lut_softmax_u8: null pointer");
    launch_begin(d);
    lut_softmax_u8_kernel<<<row_blocks(d, R), 256, 0, d->stream>>>(x, out, R, C, exp_lut, recip_lut);
    return launch_end(d, "lut_softmax_u8");
}

HX_EXPORT int hexcuda_lut_softmax_i16(int dev, const int16_t *x, int16_t *out, int R, int C,
                                     const uint16_t *exp_lut) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C < 1) return fail(HEXCUDA_ERR_ARG, "lut_softmax_i16: R %d C %d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (!x || !out || !exp_lut) return fail(HEXCUDA_ERR_ARG, "lut_softmax_i16: null pointer");
    launch_begin(d);
    lut_softmax_i16_kernel<<<row_blocks(d, R), 256, 0, d->stream>>>(x, out, R, C, exp_lut);
    return launch_end(d, "lut_softmax_i16");
}

HX_EXPORT int hexcuda_requant_i16(int dev, const int32_t *a, int16_t *out, int64_t n, int32_t mult,
                                 int shift) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0 || shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "requant_i16: n %lld shift %d", (long long)n, shift);
    if (n == 0) return HEXCUDA_OK;
    if (!a || !out) return fail(HEXCUDA_ERR_ARG, "requant_i16: null pointer");
    launch_begin(d);
    constexpr auto kern = requant_i16_kernel;
    kern<<<resident_blocks<kern>(d, n), 256, 0, d->stream>>>(a, out, n, mult, shift);
    return launch_end(d, "requant_i16");
}

HX_EXPORT int hexcuda_gate_mul_requant_i8(int dev, const int8_t *gate, const int8_t *up,
                                         const int8_t *lut, int8_t *out, int64_t n, int32_t mult,
                                         int shift) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0 || shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "gate_mul_requant_i8: n %lld shift %d", (long long)n, shift);
    if (n == 0) return HEXCUDA_OK;
    if (!gate || !up || !lut || !out) return fail(HEXCUDA_ERR_ARG, "gate_mul_requant_i8: null pointer");
    launch_begin(d);
    constexpr auto kern = gate_mul_requant_i8_kernel;
    kern<<<resident_blocks<kern>(d, n), 256, 0, d->stream>>>(gate, up, lut, out, n, mult, shift);
    return launch_end(d, "gate_mul_requant_i8");
}

HX_EXPORT int hexcuda_norm_requant_i8(int dev, const int8_t *a, int8_t *out, int64_t n, int nch,
                                     const int32_t *nmult, const int *nshift, int32_t mult,
                                     int shift, int zp) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0 || nch < 1 || shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "norm_requant_i8: n %lld channels %d shift %d", (long long)n,
                    nch, shift);
    const int64_t per_ch = n / nch;
    if (per_ch == 0) return HEXCUDA_OK;
    if (!a || !out || !nmult || !nshift) return fail(HEXCUDA_ERR_ARG, "norm_requant_i8: null pointer");
    launch_begin(d);
    constexpr auto kern = norm_requant_i8_kernel;
    kern<<<resident_blocks<kern>(d, per_ch * nch), 256, 0, d->stream>>>(a, out, n, per_ch, nch, nmult,
                                                                         nshift, mult, shift, zp);
    return launch_end(d, "norm_requant_i8");
}

// ------------------------------------------------------------- compositions
// scratch slots of the composite entries (the GEMM entries they call use 0..2)
namespace hx {
namespace {
constexpr int kSlotScores = 20, kSlotFfnHid = 21, kSlotFfnSum = 22;
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_gemm_softmax_u8(int dev, const int8_t *A, const int8_t *B, int b_transposed,
                                     const uint8_t *exp_lut, uint8_t *out, int M, int N, int K,
                                     int requant, int32_t mult, int shift) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || N < 1 || K < 0) return fail(HEXCUDA_ERR_ARG, "gemm_softmax_u8: bad shape");
    if (M == 0) return HEXCUDA_OK;
    int8_t *sc = reinterpret_cast<int8_t *>(scratch(d, kSlotScores, (size_t)M * N));
    if (!sc) return HEXCUDA_ERR_OOM;
    int rc = requant ? hexcuda_gemm_i8_rq_ex(dev, A, B, b_transposed, nullptr, nullptr, sc, M, N, K,
                                             mult, shift, 0, 0)
                     : hexcuda_gemm_i8_acc(dev, A, 1, B, b_transposed, nullptr, nullptr,
                                           HEXCUDA_HMX_RES_NONE, nullptr, sc,
                                           HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_NONE, M, N, K);
    if (rc) return rc;
    return hexcuda_lut_softmax_u8(dev, sc, out, M, N, exp_lut, nullptr);
}

HX_EXPORT int hexcuda_gelu_ffn_residual_i8(int dev, const int8_t *x, const int8_t *W1,
                                          const int32_t *b1, const int8_t *gelu_lut,
                                          const int8_t *W2, const int32_t *b2, const int8_t *x_res,
                                          const int8_t *gamma, const int8_t *beta,
                                          const uint8_t *inv_lut, int8_t *out, int M, int K, int V,
                                          int D) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (M < 0 || K < 0 || V < 0 || D < 1) return fail(HEXCUDA_ERR_ARG, "gelu_ffn_residual_i8: bad shape");
    if (M == 0) return HEXCUDA_OK;
    int8_t *hid = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnHid, (size_t)M * (V > 0 ? V : 1)));
    int8_t *sum = reinterpret_cast<int8_t *>(scratch(d, kSlotFfnSum, (size_t)M * D));
    if (!hid || !sum) return HEXCUDA_ERR_OOM;
    if (V > 0) {
        if (int rc = hexcuda_gemm_i8_acc(dev, x, 1, W1, 0, b1, nullptr, HEXCUDA_HMX_RES_NONE, gelu_lut,
                                         hid, HEXCUDA_HMX_STORE_LUT_I8, HEXCUDA_HMX_ACT_NONE, M, V, K))
            return rc;
    }
    if (int rc = hexcuda_gemm_i8_acc(dev, hid, 1, W2, 0, b2, x_res, HEXCUDA_HMX_RES_I8, nullptr, sum,
                                     HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_NONE, M, D, V))
        return rc;
    return hexcuda_layernorm_lut_i8(dev, sum, nullptr, nullptr, out, M, D, gamma, beta, inv_lut,
                                    HEXCUDA_LN_AFFINE_SHARED);
}
