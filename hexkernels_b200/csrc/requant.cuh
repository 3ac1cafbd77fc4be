// requant.cuh -- the corpus's fixed-point requant arithmetic on the device.
//
//   v = (int64) x * mult
//   half = shift > 0 ? 1 << (shift - 1) : 0
//   r = v >= 0 ? (v + half) >> shift : -((-v + half) >> shift)
//   out = saturate(r + zp)
//
// kernels/expert/i8_gemm_requant/reference.c:11-16,
// requant_per_channel/reference.c:7-13, requantize_i32_u8_dma/reference.c:6-11.
// shift is clamped to 63 (the C reference is undefined beyond that).
#pragma once
#include <stdint.h>

namespace hx {

__device__ __forceinline__ int64_t rq_round(int64_t v, int shift) {
    shift = shift < 0 ? 0 : (shift > 63 ? 63 : shift);
    const int64_t half = shift > 0 ? ((int64_t)1 << (shift - 1)) : 0;
    return v >= 0 ? ((v + half) >> shift) : -(((-v) + half) >> shift);
}

__device__ __forceinline__ int requant_i8(int64_t x, int32_t mult, int shift, int zp) {
    int64_t r = rq_round(x * (int64_t)mult, shift) + zp;
    r = r > 127 ? 127 : r;
    r = r < -128 ? -128 : r;
    return (int)r;
}

__device__ __forceinline__ uint32_t requant_u8(int64_t x, int32_t mult, int shift, int zp) {
    int64_t r = rq_round(x * (int64_t)mult, shift) + zp;
    r = r > 255 ? 255 : r;
    r = r < 0 ? 0 : r;
    return (uint32_t)r;
}

}  // namespace hx
