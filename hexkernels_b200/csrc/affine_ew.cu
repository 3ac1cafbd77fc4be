// affine_ew.cu -- the integer affine elementwise family of the requant
// epilogues that the requant_ew kernel's int32 / int8 inputs and
// round-half-away-only rounding do not cover:
//
//   out[i] = clamp(round((x[i] - zp_in) * mult + add, shift) + zp_out, lo, hi)
//
// x int8, uint8, int16 or int32; out int8, uint8, int16 or int32; round
// either half away from zero on the sign-magnitude value or the plain
// arithmetic right shift (floor); wrap32 takes the product and sum modulo
// 2^32 first, as the references' int32 arithmetic does, else they are exact
// in int64.  Callers (kernels/expert/<name>/reference.c):
//   rescale_i16_i8_dma    int16 x 3, half away >> 4, int8        (:5-15)
//   dequant_i8_i16_dma    (x - zp) * scale >> shift (floor), int16 (:5-12)
//   hmx_requant_store_i8  (acc * 17 + 8) >> 4 (floor), int8      (:3-8)
//   i8_add_bias_sat_dma   x + bias, int8                          (:3-9)
//   i8_element_affine_dma x * scale + shift, half away >> s, int8 (:5-16)
// HBM-bound: 16 elements per thread step, grid sized by occupancy.
#include "ew_launch.cuh"
#include "hx_internal.h"

namespace hx {
namespace {

struct AffineArgs {
    int32_t zp_in, mult;
    int64_t add;
    int shift, wrap32, zp_out;
    int32_t lo, hi;
};

template <int ELEM> struct ElemT;
template <> struct ElemT<HEXCUDA_ELEM_I8> { using T = int8_t; };
template <> struct ElemT<HEXCUDA_ELEM_U8> { using T = uint8_t; };
template <> struct ElemT<HEXCUDA_ELEM_I16> { using T = int16_t; };
template <> struct ElemT<HEXCUDA_ELEM_I32> { using T = int32_t; };

template <bool FLOOR>
__device__ __forceinline__ int64_t affine_one(int64_t x, const AffineArgs &a) {
    int64_t v;
    if (a.wrap32)
        v = (int64_t)(int32_t)(((uint32_t)(int32_t)x - (uint32_t)a.zp_in) * (uint32_t)a.mult +
                               (uint32_t)a.add);
    else
        v = (x - a.zp_in) * (int64_t)a.mult + a.add;
    int64_t r;
    if (FLOOR) {
        r = v >> a.shift;
    } else {
        const int64_t half = a.shift > 0 ? ((int64_t)1 << (a.shift - 1)) : 0;
        r = v >= 0 ? ((v + half) >> a.shift) : -(((-v) + half) >> a.shift);
    }
    r += a.zp_out;
    return r < a.lo ? a.lo : (r > a.hi ? a.hi : r);
}

template <int EI, int EO, bool FLOOR>
__global__ void __launch_bounds__(256) affine_ew_kernel(const void *__restrict__ in,
                                                        void *__restrict__ out, int64_t n,
                                                        const AffineArgs a) {
    using TI = typename ElemT<EI>::T;
    using TO = typename ElemT<EO>::T;
    const TI *x = reinterpret_cast<const TI *>(in);
    TO *y = reinterpret_cast<TO *>(out);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x * 16;
    for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 16; base < n;
         base += stride) {
        if (base + 16 <= n) {
            TI v[16];
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = __ldcs(x + base + k);
#pragma unroll
            for (int k = 0; k < 16; k++) y[base + k] = (TO)affine_one<FLOOR>((int64_t)v[k], a);
        } else {
            for (int64_t i = base; i < n; i++) y[i] = (TO)affine_one<FLOOR>((int64_t)x[i], a);
        }
    }
}

template <int EI, int EO>
int affine_launch_out(Dev *d, const void *in, void *out, int64_t n, const AffineArgs &a, bool floor_) {
    if (floor_) {
        constexpr auto kern = affine_ew_kernel<EI, EO, true>;
        kern<<<resident_blocks<kern>(d, (n + 15) / 16), 256, 0, d->stream>>>(in, out, n, a);
    } else {
        constexpr auto kern = affine_ew_kernel<EI, EO, false>;
        kern<<<resident_blocks<kern>(d, (n + 15) / 16), 256, 0, d->stream>>>(in, out, n, a);
    }
    return HEXCUDA_OK;
}

template <int EI>
int affine_launch(Dev *d, const void *in, void *out, int eo, int64_t n, const AffineArgs &a,
                  bool floor_) {
    switch (eo) {
    case HEXCUDA_ELEM_I8: return affine_launch_out<EI, HEXCUDA_ELEM_I8>(d, in, out, n, a, floor_);
    case HEXCUDA_ELEM_U8: return affine_launch_out<EI, HEXCUDA_ELEM_U8>(d, in, out, n, a, floor_);
    case HEXCUDA_ELEM_I16: return affine_launch_out<EI, HEXCUDA_ELEM_I16>(d, in, out, n, a, floor_);
    default: return affine_launch_out<EI, HEXCUDA_ELEM_I32>(d, in, out, n, a, floor_);
    }
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_affine_ew(int dev, const void *in, int elem_in, void *out, int elem_out,
                                int64_t n, int32_t zp_in, int32_t mult, int64_t add, int shift,
                                int round, int wrap32, int zp_out, int32_t lo, int32_t hi) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (elem_in < HEXCUDA_ELEM_I8 || elem_in > HEXCUDA_ELEM_I32 || elem_out < HEXCUDA_ELEM_I8 ||
        elem_out > HEXCUDA_ELEM_I32 || n < 0 || shift < 0 || shift > (wrap32 ? 31 : 62) ||
        (round != HEXCUDA_ROUND_HALF_AWAY && round != HEXCUDA_ROUND_FLOOR) || lo > hi ||
        (!wrap32 && (add > ((int64_t)1 << 62) || add < -((int64_t)1 << 62))))
        return fail(HEXCUDA_ERR_ARG, "affine_ew: elem %d -> %d n %lld shift %d round %d lo %d hi %d",
                    elem_in, elem_out, (long long)n, shift, round, lo, hi);
    if (n == 0) return HEXCUDA_OK;
    if (!in || !out) return fail(HEXCUDA_ERR_ARG, "affine_ew: null pointer");
    const AffineArgs a{zp_in, mult, add, shift, wrap32 ? 1 : 0, zp_out, lo, hi};
    const bool fl = round == HEXCUDA_ROUND_FLOOR;
    launch_begin(d);
    switch (elem_in) {
    case HEXCUDA_ELEM_I8: affine_launch<HEXCUDA_ELEM_I8>(d, in, out, elem_out, n, a, fl); break;
    case HEXCUDA_ELEM_U8: affine_launch<HEXCUDA_ELEM_U8>(d, in, out, elem_out, n, a, fl); break;
    case HEXCUDA_ELEM_I16: affine_launch<HEXCUDA_ELEM_I16>(d, in, out, elem_out, n, a, fl); break;
    default: affine_launch<HEXCUDA_ELEM_I32>(d, in, out, elem_out, n, a, fl); break;
    }
    return launch_end(d, "affine_ew");
}
