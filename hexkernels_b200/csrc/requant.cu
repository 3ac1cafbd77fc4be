// requant.cu -- standalone int32 -> int8 / uint8 fixed-point requant kernels
// (HBM-bound streaming) and the shared requant arithmetic.
//
// Requant (kernels/expert/requant_per_channel/reference.c:7-14 and
// requantize_i32_u8_dma/reference.c:5-13):
//     v = (int64) a * mult
//     r = v >= 0 ? (v + half) >> shift : -((-v + half) >> shift),
//         half = shift > 0 ? 1 << (shift - 1) : 0     (round half away from 0)
//     out = saturate(r + zp)
// All integer, so the device result is bit-identical to the reference.
#include "hx_internal.h"
#include "requant.cuh"

namespace hx {
namespace {

// Each thread converts 16 consecutive int32 (four 128-bit loads) into 16
// bytes (one 128-bit store); a scalar tail handles n % 16 and misalignment.
__global__ void __launch_bounds__(256) requantize_i32_u8_kernel(const int32_t *__restrict__ a,
                                                                 uint8_t *__restrict__ out,
                                                                 int64_t n, int32_t mult,
                                                                 int shift, int zp, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t nv = n / 16;
        for (int64_t v = t; v < nv; v += stride) {
            const int4 *src = reinterpret_cast<const int4 *>(a) + v * 4;
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int4 x = __ldcs(src + q);
                uint32_t b0 = requant_u8(x.x, mult, shift, zp);
                uint32_t b1 = requant_u8(x.y, mult, shift, zp);
                uint32_t b2 = requant_u8(x.z, mult, shift, zp);
                uint32_t b3 = requant_u8(x.w, mult, shift, zp);
                w[q] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
            }
            __stcs(reinterpret_cast<uint4 *>(out) + v, make_uint4(w[0], w[1], w[2], w[3]));
        }
        for (int64_t i = nv * 16 + t; i < n; i += stride) out[i] = requant_u8(a[i], mult, shift, zp);
    } else {
        for (int64_t i = t; i < n; i += stride) out[i] = requant_u8(a[i], mult, shift, zp);
    }
}

// Per-channel: row r uses mult[r], shift[r].  One CTA row-strip per row
// chunk; 4 elements per thread step.
__global__ void __launch_bounds__(256) requant_per_channel_kernel(
    const int32_t *__restrict__ a, int8_t *__restrict__ out, int R, int C,
    const int32_t *__restrict__ mult, const int *__restrict__ shift, int zp) {
    for (int r = blockIdx.y; r < R; r += gridDim.y) {
        const int32_t m = mult[r];
        const int s = shift[r];
        const int32_t *ar = a + (size_t)r * C;
        int8_t *orow = out + (size_t)r * C;
        for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x)
            orow[c] = requant_i8(ar[c], m, s, zp);
    }
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_requantize_i32_u8(int dev, const int32_t *a, uint8_t *out, int64_t n,
                                        int32_t mult, int shift, uint8_t zp) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0 || shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "requantize_i32_u8: n=%lld shift=%d (0..63)", (long long)n,
                    shift);
    if (n == 0) return HEXCUDA_OK;
    if (!a || !out) return fail(HEXCUDA_ERR_ARG, "requantize_i32_u8: null pointer");
    int vec = (((uintptr_t)a & 15u) == 0) && (((uintptr_t)out & 15u) == 0);
    int64_t work = vec ? (n + 15) / 16 : n;
    int64_t blocks = (work + 255) / 256;
    int64_t cap = (int64_t)d->sms * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    launch_begin(d);
    requantize_i32_u8_kernel<<<(unsigned)blocks, 256, 0, d->stream>>>(a, out, n, mult, shift,
                                                                       (int)zp, vec);
    return launch_end(d, "requantize_i32_u8");
}

HX_EXPORT int hexcuda_requant_per_channel(int dev, const int32_t *a, int8_t *out, int R, int C,
                                          const int32_t *mult, const int *shift, int8_t zp) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C < 0) return fail(HEXCUDA_ERR_ARG, "requant_per_channel: R=%d C=%d", R, C);
    if (R == 0 || C == 0) return HEXCUDA_OK;
    if (!a || !out || !mult || !shift)
        return fail(HEXCUDA_ERR_ARG, "requant_per_channel: null pointer");
    unsigned gx = (unsigned)((C + 255) / 256);
    if (gx > 64) gx = 64;
    unsigned gy = (unsigned)(R < 65535 ? R : 65535);
    launch_begin(d);
    requant_per_channel_kernel<<<dim3(gx, gy), 256, 0, d->stream>>>(a, out, R, C, mult, shift,
                                                                     (int)zp);
    return launch_end(d, "requant_per_channel");
}
