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
#include "ew_launch.cuh"

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

// ---------------------------------------------------------------------------
// Elementwise requant family: x = pre(a, b); r = requant(x) + zp; two clamps;
// out = lut ? lut[(uint8) r] : (uint8) r.  (The corpus bundles it covers are
// listed with hexcuda_requant_ew in hexcuda.h.)
struct RqEw {
    int pre;            // HEXCUDA_RQ_PRE_*
    int64_t c;          // MUL_ADD constant
    int32_t mult;
    int shift;          // 0..63
    int zp;
    int sign_of_a;      // sign(x) * ((|x| * mult + half) >> shift)
    int lo1, hi1, lo2, hi2;
    const int8_t *lut;  // 256 entries or null
    int lo, hi;         // the two clamps folded into one (set by the entry)
    uint32_t amult;     // |mult|
    bool mneg;          // mult < 0
    int lo_z, hi_z;     // lo - zp, hi - zp
};

// One element.  PRE, SIGN_OF_A and SHIFT_HI (shift >= 32) are compile-time
// so the per-element code has no mode branches; the kernel is bound by the
// integer ALU pipe, so the common forms work on 32-bit words:
//  * pre(a, b) for A / ADD / ADD_RELU is at most 33 bits; its magnitude fits
//    32 bits except x = -2^32, which takes the general path;
//  * |x| * |mult| + half is one 32 x 32 -> 64 multiply-add, and with shift
//    >= 32 the reference's arithmetic shift of that int64 (including its
//    wrap past 2^63 at the largest shifts) is a 32-bit shift of the high word;
//  * magnitudes beyond 2^28 (or below -2^28 after a wrap) saturate every
//    clamp (zp, lo and hi are within +-2^24, checked by the entry), so only
//    the lower cap is applied before the sign and the clamp runs as
//    clamp(r, lo - zp, hi - zp) + zp.
// p.lo / p.hi are the two clamps folded into one (the composition of two
// clamps is the clamp to [clamp(lo1, lo2, hi2), clamp(hi1, lo2, hi2)]).
template <int PRE, bool SIGN_OF_A, bool SHIFT_HI>
__device__ __forceinline__ uint32_t rq_ew_one(int32_t a, int32_t b, const RqEw &p, int64_t half) {
    constexpr int kCap = 1 << 28;
    int32_t r32;
    bool general = SIGN_OF_A || PRE == HEXCUDA_RQ_PRE_MUL_ADD;
    if constexpr (!SIGN_OF_A && PRE != HEXCUDA_RQ_PRE_MUL_ADD) {
        uint32_t lo;
        bool xneg;
        if constexpr (PRE == HEXCUDA_RQ_PRE_A) {
            xneg = a < 0;
            lo = (uint32_t)a;
        } else {
            const int64_t x = (int64_t)a + b;
            lo = (uint32_t)x;
            xneg = x < 0;
            if constexpr (PRE == HEXCUDA_RQ_PRE_ADD_RELU) {
                if (xneg) lo = 0;
                xneg = false;
            } else {
                general = xneg && lo == 0;      // x = -2^32
            }
        }
        const uint32_t ax = xneg ? 0u - lo : lo;
        const uint64_t t = (uint64_t)ax * p.amult + (uint64_t)half;
        int32_t ra;
        if constexpr (SHIFT_HI) {
            ra = max((int32_t)(uint32_t)(t >> 32) >> (p.shift - 32), -kCap);
        } else {
            const int64_t r = (int64_t)t >> p.shift;
            ra = (int32_t)(r > kCap ? kCap : (r < -kCap ? -kCap : r));
        }
        r32 = (xneg != p.mneg) ? -ra : ra;
    }
    if (general) {
        int64_t x = a;
        if constexpr (PRE == HEXCUDA_RQ_PRE_ADD || PRE == HEXCUDA_RQ_PRE_ADD_RELU) {
            x = (int64_t)a + b;
        } else if constexpr (PRE == HEXCUDA_RQ_PRE_MUL_ADD) {
            x = (int64_t)((uint64_t)(int64_t)a * (uint64_t)(int64_t)b + (uint64_t)p.c);
        }
        int64_t r;
        if (SIGN_OF_A) {
            const bool xneg = x < 0;
            const uint64_t ax = xneg ? 0ull - (uint64_t)x : (uint64_t)x;
            const int64_t am = (int64_t)(ax * (uint64_t)(int64_t)p.mult);
            const int64_t sh = (am + half) >> p.shift;
            r = xneg ? -sh : sh;
        } else {
            r = rq_round((int64_t)((uint64_t)x * (uint64_t)(int64_t)p.mult), p.shift);
        }
        r32 = (int32_t)(r > kCap ? kCap : (r < -kCap ? -kCap : r));
    }
    r32 = max(min(r32, p.hi_z), p.lo_z) + p.zp;
    if (p.lut) return (uint32_t)(uint8_t)__ldg(p.lut + (uint8_t)r32);
    return (uint32_t)r32 & 0xFFu;
}

// four results (low bytes) into one 32-bit word
__device__ __forceinline__ uint32_t pack4(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
    return __byte_perm(__byte_perm(x0, x1, 0x0040), __byte_perm(x2, x3, 0x0040), 0x5410);
}

// 16 consecutive elements of one operand as int64 (int8 or int32 source)
template <bool I8>
__device__ __forceinline__ void load16(const void *src, int64_t v, int32_t (&x)[16]) {
    if constexpr (I8) {
        const uint4 q = __ldcs(reinterpret_cast<const uint4 *>(src) + v);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 16; i++) x[i] = (int8_t)(w[i >> 2] >> (8 * (i & 3)));
    } else {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int4 q = __ldcs(reinterpret_cast<const int4 *>(src) + v * 4 + k);
            x[4 * k] = q.x, x[4 * k + 1] = q.y, x[4 * k + 2] = q.z, x[4 * k + 3] = q.w;
        }
    }
}

template <bool I8>
__device__ __forceinline__ int32_t load1(const void *src, int64_t i) {
    if constexpr (I8)
        return reinterpret_cast<const int8_t *>(src)[i];
    else
        return reinterpret_cast<const int32_t *>(src)[i];
}

// 4 consecutive elements of one operand (int32: one 16-byte load; int8:
// one 4-byte load); consecutive lanes read consecutive 4-element groups, so
// every load instruction of a warp is one contiguous run.
template <bool I8>
__device__ __forceinline__ void load4(const void *src, int64_t v, int32_t (&x)[4]) {
    if constexpr (I8) {
        const uint32_t w = __ldcs(reinterpret_cast<const unsigned int *>(src) + v);
#pragma unroll
        for (int i = 0; i < 4; i++) x[i] = (int8_t)(w >> (8 * i));
    } else {
        const int4 q = __ldcs(reinterpret_cast<const int4 *>(src) + v);
        x[0] = q.x, x[1] = q.y, x[2] = q.z, x[3] = q.w;
    }
}

// Six blocks per SM (at most 40 registers a thread): the loads in flight of
// 48 warps, against 40 at the register count ptxas picks unbounded; eight
// blocks (32 registers) spill.
template <bool A_I8, int B_KIND, int PRE, bool SIGN_OF_A, bool SHIFT_HI>
__global__ void __launch_bounds__(256, 6) requant_ew_kernel(const void *__restrict__ a,
                                                          const void *__restrict__ b,
                                                          uint8_t *__restrict__ out, int64_t n,
                                                          const RqEw p, int vec) {
    const int64_t half = p.shift > 0 ? ((int64_t)1 << (p.shift - 1)) : 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    constexpr bool kWide = A_I8 && B_KIND != 1;   // int8 data only: 16 per step
    int64_t done = 0;
    if (vec && kWide) {
        const int64_t nv = n / 16;
        for (int64_t v = t; v < nv; v += stride) {
            int32_t xa[16], xb[16];
            load16<true>(a, v, xa);
            if constexpr (B_KIND != 0) load16<true>(b, v, xb);
            uint32_t y[16], w[4];
#pragma unroll
            for (int i = 0; i < 16; i++)
                y[i] = rq_ew_one<PRE, SIGN_OF_A, SHIFT_HI>(xa[i], B_KIND != 0 ? xb[i] : 0, p, half);
#pragma unroll
            for (int k = 0; k < 4; k++) w[k] = pack4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
            __stcs(reinterpret_cast<uint4 *>(out) + v, make_uint4(w[0], w[1], w[2], w[3]));
        }
        done = nv * 16;
    } else if (vec) {
        // two grid-stride steps per iteration: both steps' loads are issued
        // before any result is needed (memory-level parallelism)
        const int64_t nv = n / 4;
        int64_t v = t;
        for (; v + stride < nv; v += 2 * stride) {
            int32_t xa[2][4], xb[2][4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                load4<A_I8>(a, v + u * stride, xa[u]);
                if constexpr (B_KIND != 0) load4<B_KIND == 2>(b, v + u * stride, xb[u]);
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                uint32_t y[4];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    y[i] = rq_ew_one<PRE, SIGN_OF_A, SHIFT_HI>(xa[u][i], B_KIND != 0 ? xb[u][i] : 0, p, half);
                __stcs(reinterpret_cast<unsigned int *>(out) + v + u * stride, pack4(y[0], y[1], y[2], y[3]));
            }
        }
        for (; v < nv; v += stride) {
            int32_t xa[4], xb[4];
            load4<A_I8>(a, v, xa);
            if constexpr (B_KIND != 0) load4<B_KIND == 2>(b, v, xb);
            uint32_t y[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                y[i] = rq_ew_one<PRE, SIGN_OF_A, SHIFT_HI>(xa[i], B_KIND != 0 ? xb[i] : 0, p, half);
            __stcs(reinterpret_cast<unsigned int *>(out) + v, pack4(y[0], y[1], y[2], y[3]));
        }
        done = nv * 4;
    }
    for (int64_t i = done + t; i < n; i += stride) {
        const int32_t bi = B_KIND == 0 ? 0 : load1<B_KIND == 2>(b, i);
        out[i] = (uint8_t)rq_ew_one<PRE, SIGN_OF_A, SHIFT_HI>(load1<A_I8>(a, i), bi, p, half);
    }
}

// out[r][c] = acc[r][c] + bias[c] (int32, wrap): 4 columns per thread step
__global__ void __launch_bounds__(256) epilogue_bias_i32_kernel(const int32_t *__restrict__ acc,
                                                                 const int32_t *__restrict__ bias,
                                                                 int32_t *__restrict__ out, int R,
                                                                 int C, int vec) {
    const int64_t total = (int64_t)R * C;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {  // C % 4 == 0 and 16-byte aligned buffers
        for (int64_t v = t; v < total / 4; v += stride) {
            const int c = (int)((v * 4) % C);
            const int4 x = __ldcs(reinterpret_cast<const int4 *>(acc) + v);
            const int4 bb = __ldg(reinterpret_cast<const int4 *>(bias + c));
            __stcs(reinterpret_cast<int4 *>(out) + v,
                   make_int4((int)((uint32_t)x.x + (uint32_t)bb.x), (int)((uint32_t)x.y + (uint32_t)bb.y),
                             (int)((uint32_t)x.z + (uint32_t)bb.z), (int)((uint32_t)x.w + (uint32_t)bb.w)));
        }
    } else {
        for (int64_t i = t; i < total; i += stride)
            out[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)bias[i % C]);
    }
}

// out = max(x, 0) on int8, 16 per thread step
__global__ void __launch_bounds__(256) relu_i8_kernel(const int8_t *__restrict__ x,
                                                       int8_t *__restrict__ out, int64_t n, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        for (int64_t v = t; v < n / 16; v += stride) {
            const uint4 q = __ldcs(reinterpret_cast<const uint4 *>(x) + v);
            uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 4; k++) w[k] = __vmaxs4(w[k], 0u);
            __stcs(reinterpret_cast<uint4 *>(out) + v, make_uint4(w[0], w[1], w[2], w[3]));
        }
        done = n / 16 * 16;
    }
    for (int64_t i = done + t; i < n; i += stride) out[i] = x[i] > 0 ? x[i] : 0;
}

template <bool A_I8, int B_KIND, int PRE, bool SIGN_OF_A>
void launch_rq_ew(const Dev *d, int64_t work, const void *a, const void *b, uint8_t *o, int64_t n,
                  const RqEw &p, int vec) {
    constexpr bool kFast = !SIGN_OF_A && PRE != HEXCUDA_RQ_PRE_MUL_ADD;
    if (kFast && p.shift >= 32) {
        constexpr auto kern = requant_ew_kernel<A_I8, B_KIND, PRE, SIGN_OF_A, kFast>;
        kern<<<resident_blocks<kern>(d, work), 256, 0, d->stream>>>(a, b, o, n, p, vec);
    } else {
        constexpr auto kern = requant_ew_kernel<A_I8, B_KIND, PRE, SIGN_OF_A, false>;
        kern<<<resident_blocks<kern>(d, work), 256, 0, d->stream>>>(a, b, o, n, p, vec);
    }
}

int ew_blocks(const Dev *d, int64_t work) {
    int64_t blocks = (work + 255) / 256;
    const int64_t cap = (int64_t)d->sms * 8;
    if (blocks > cap) blocks = cap;
    return blocks < 1 ? 1 : (int)blocks;
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
    if (vec) note_mech(kMechVec128);
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

HX_EXPORT int hexcuda_requant_ew(int dev, const void *a, int a_i8, const void *b, int b_kind,
                                 void *out, int64_t n, int pre, int64_t pre_c, int32_t mult,
                                 int shift, int zp, int sign_of_a, int lo1, int hi1, int lo2,
                                 int hi2, const int8_t *lut) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    const int kLim = 1 << 24;
    if (zp < -kLim || zp > kLim || lo1 < -kLim || lo1 > kLim || hi1 < -kLim || hi1 > kLim ||
        lo2 < -kLim || lo2 > kLim || hi2 < -kLim || hi2 > kLim)
        return fail(HEXCUDA_ERR_ARG, "requant_ew: zp / clamp bounds beyond +-2^24");
    if (n < 0 || shift < 0 || shift > 63 || b_kind < 0 || b_kind > 2 ||
        pre < HEXCUDA_RQ_PRE_A || pre > HEXCUDA_RQ_PRE_MUL_ADD || (pre != HEXCUDA_RQ_PRE_A && !b_kind))
        return fail(HEXCUDA_ERR_ARG, "requant_ew: n=%lld shift=%d b_kind=%d pre=%d", (long long)n,
                    shift, b_kind, pre);
    if (n == 0) return HEXCUDA_OK;
    if (!a || !out || (b_kind && !b)) return fail(HEXCUDA_ERR_ARG, "requant_ew: null pointer");
    RqEw p{pre, pre_c, mult, shift, zp, sign_of_a ? 1 : 0, lo1, hi1, lo2, hi2, lut, 0, 0, 0, false, 0, 0};
    {
        auto clampi = [](int v, int lo, int hi) { return std::max(std::min(v, hi), lo); };
        p.lo = clampi(lo1, lo2, hi2);
        p.hi = clampi(hi1, lo2, hi2);
        p.amult = mult < 0 ? 0u - (uint32_t)mult : (uint32_t)mult;
        p.mneg = mult < 0;
        p.lo_z = p.lo - zp;
        p.hi_z = p.hi - zp;
    }
    auto al = [](const void *q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
    const int vec = al(a) && al(b) && al(out);
    const int per = (a_i8 && b_kind != 1) ? 16 : 4;
    const int64_t work = vec ? (n + per - 1) / per : n;
    uint8_t *o = reinterpret_cast<uint8_t *>(out);
    launch_begin(d);
    if (sign_of_a) {
        if (pre != HEXCUDA_RQ_PRE_A) return fail(HEXCUDA_ERR_ARG, "requant_ew: sign_of_a takes a alone");
        if (a_i8)
            launch_rq_ew<true, 0, HEXCUDA_RQ_PRE_A, true>(d, work, a, b, o, n, p, vec);
        else
            launch_rq_ew<false, 0, HEXCUDA_RQ_PRE_A, true>(d, work, a, b, o, n, p, vec);
    } else if (pre == HEXCUDA_RQ_PRE_A) {
        if (a_i8)
            launch_rq_ew<true, 0, HEXCUDA_RQ_PRE_A, false>(d, work, a, b, o, n, p, vec);
        else
            launch_rq_ew<false, 0, HEXCUDA_RQ_PRE_A, false>(d, work, a, b, o, n, p, vec);
    } else {
        // two-operand forms: int32 pairs or int8 pairs (the corpus's bundles)
        if (a_i8 != (b_kind == 2))
            return fail(HEXCUDA_ERR_ARG, "requant_ew: a and b must both be int32 or both int8");
#define HX_RQ2(P)                                                                                 \
    if (a_i8)                                                                                    \
        launch_rq_ew<true, 2, P, false>(d, work, a, b, o, n, p, vec); \
    else                                                                                         \
        launch_rq_ew<false, 1, P, false>(d, work, a, b, o, n, p, vec);
        if (pre == HEXCUDA_RQ_PRE_ADD) {
            HX_RQ2(HEXCUDA_RQ_PRE_ADD)
        } else if (pre == HEXCUDA_RQ_PRE_ADD_RELU) {
            HX_RQ2(HEXCUDA_RQ_PRE_ADD_RELU)
        } else {
            HX_RQ2(HEXCUDA_RQ_PRE_MUL_ADD)
        }
#undef HX_RQ2
    }
    if (vec) note_mech(kMechVec128);
    return launch_end(d, "requant_ew");
}

HX_EXPORT int hexcuda_epilogue_bias_i32(int dev, const int32_t *acc, const int32_t *bias,
                                        int32_t *out, int R, int C) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C < 0) return fail(HEXCUDA_ERR_ARG, "epilogue_bias_i32: R=%d C=%d", R, C);
    if (R == 0 || C == 0) return HEXCUDA_OK;
    if (!acc || !bias || !out) return fail(HEXCUDA_ERR_ARG, "epilogue_bias_i32: null pointer");
    auto al = [](const void *q) { return ((uintptr_t)q & 15u) == 0; };
    const int vec = (C % 4 == 0) && al(acc) && al(bias) && al(out);
    const int64_t total = (int64_t)R * C;
    launch_begin(d);
    epilogue_bias_i32_kernel<<<ew_blocks(d, vec ? total / 4 : total), 256, 0, d->stream>>>(
        acc, bias, out, R, C, vec);
    return launch_end(d, "epilogue_bias_i32");
}

HX_EXPORT int hexcuda_relu_i8(int dev, const int8_t *x, int8_t *out, int64_t n) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "relu_i8: n=%lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (!x || !out) return fail(HEXCUDA_ERR_ARG, "relu_i8: null pointer");
    const int vec = (((uintptr_t)x | (uintptr_t)out) & 15u) == 0;
    launch_begin(d);
    relu_i8_kernel<<<ew_blocks(d, vec ? (n + 15) / 16 : n), 256, 0, d->stream>>>(x, out, n, vec);
    return launch_end(d, "relu_i8");
}
