// reduce_int.cu -- integer whole-array reductions and their elementwise
// neighbours, HBM-bound streaming kernels:
//   hexcuda_reduce_int            sum / int64 sum / sum of squares / squared
//                                 difference / dot / L1 / absmax / max / min /
//                                 argmax / argmin / top-1 / mean
//   hexcuda_minmax_ew             elementwise max / min, two arrays or a scalar
//   hexcuda_group_sum_i8          sums of w consecutive int8
//   hexcuda_scan_max_i8           inclusive prefix maximum
//   hexcuda_head_group_reduce_i8  sum of a group's head planes + requant
// The semantics are those of kernels/expert/<bundle>/reference.c for
// vtcm_reduce_i32, i8_sum_dma, dma_double_buffer_reduce_i32, i8_sumsq_i32,
// i8_sumsq_diff_i32, i8_weighted_sum, i8_l1norm_dma, i8_absmax_dma,
// dma_stream_max_u8, i8_argmax_dma, i8_argmin_dma, i8_top1_reduce_dma,
// i8_mean_dma, hvx_vmax_i8, hvx_vmax_u8, hvx_vmin_i16, hvx_vmin_u8,
// i8_max_scalar_dma, i8_min_scalar_dma, hvx_vradd_i8_reduce, i8_scan_max and
// gqa_group_reduce_i8.
//
// The references' int32 accumulators wrap modulo 2^32 and wrapping addition
// is associative, so any order of partial sums gives the same bits: threads
// accumulate in uint32 (dp4a for the byte forms, four values or products per
// instruction) and partials combine modulo 2^32; the int64 sum accumulates in
// int64 throughout.  Arg reductions carry (value, first index) pairs: a larger
// (smaller) value wins, an equal value keeps the smaller index, which is the
// references' left-to-right scan with a strict comparison.
#include <limits.h>

#include <algorithm>
#include <vector>

#include "ew_launch.cuh"
#include "hx_internal.h"
#include "requant.cuh"

namespace hx {
namespace {

constexpr int kSlotRedPart = 16;   // per-block partials
constexpr int kSlotRedOne = 17;    // one combined partial / scan block maxima
constexpr int kSlotScanCarry = 18; // scan carries

struct RedPart {
    long long v;     // sum (mod 2^32, or int64 for SUM64) or extreme value
    long long i;     // first index of the extreme value (arg reductions)
};

__host__ __device__ constexpr bool red_arg(int op) {
    return op == HEXCUDA_RED_ARGMAX || op == HEXCUDA_RED_ARGMIN || op == HEXCUDA_RED_TOP1;
}
__host__ __device__ constexpr bool red_ext(int op) {
    return op == HEXCUDA_RED_ABSMAX || op == HEXCUDA_RED_MAX || op == HEXCUDA_RED_MIN || red_arg(op);
}
__host__ __device__ constexpr bool red_min(int op) {
    return op == HEXCUDA_RED_MIN || op == HEXCUDA_RED_ARGMIN;
}
__host__ __device__ constexpr bool red_needs_b(int op) {
    return op == HEXCUDA_RED_SUMSQ_DIFF || op == HEXCUDA_RED_DOT;
}

template <int OP>
__host__ __device__ __forceinline__ RedPart red_identity() {
    if constexpr (!red_ext(OP)) return RedPart{0, 0};
    else if constexpr (red_min(OP)) return RedPart{LLONG_MAX, LLONG_MAX};
    else return RedPart{LLONG_MIN, LLONG_MAX};
}

template <int OP>
__host__ __device__ __forceinline__ RedPart red_combine(RedPart x, RedPart y) {
    if constexpr (OP == HEXCUDA_RED_SUM64) {
        return RedPart{(long long)((unsigned long long)x.v + (unsigned long long)y.v), 0};
    } else if constexpr (!red_ext(OP)) {
        return RedPart{(long long)(uint32_t)((uint32_t)x.v + (uint32_t)y.v), 0};
    } else if constexpr (red_min(OP)) {
        return (y.v < x.v || (y.v == x.v && y.i < x.i)) ? y : x;
    } else {
        return (y.v > x.v || (y.v == x.v && y.i < x.i)) ? y : x;
    }
}

// the op's result from the combined partial of all n elements
template <int OP>
__host__ __device__ __forceinline__ void red_write(RedPart p, int64_t n, void *out) {
    int32_t *o32 = reinterpret_cast<int32_t *>(out);
    if constexpr (OP == HEXCUDA_RED_SUM64) {
        *reinterpret_cast<int64_t *>(out) = (int64_t)p.v;
    } else if constexpr (OP == HEXCUDA_RED_MEAN) {
        *o32 = (int32_t)((int64_t)(int32_t)(uint32_t)p.v / n);   // C: int / int truncates
    } else if constexpr (!red_ext(OP)) {
        *o32 = (int32_t)(uint32_t)p.v;
    } else if constexpr (OP == HEXCUDA_RED_TOP1) {
        o32[0] = (int32_t)p.v;
        o32[1] = (int32_t)p.i;
    } else if constexpr (red_arg(OP)) {
        *o32 = (int32_t)p.i;
    } else {
        *o32 = n == 0 ? 0 : (int32_t)p.v;   // empty MAX / MIN / ABSMAX: 0
    }
}

template <int OP>
__device__ __forceinline__ RedPart red_warp(RedPart p) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        RedPart q;
        q.v = __shfl_down_sync(0xffffffffu, p.v, o);
        q.i = __shfl_down_sync(0xffffffffu, p.i, o);
        p = red_combine<OP>(p, q);
    }
    return p;
}

// block of 256 threads -> thread 0 holds the block's partial
template <int OP>
__device__ __forceinline__ RedPart red_block(RedPart p) {
    __shared__ RedPart ws[8];
    p = red_warp<OP>(p);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = p;
    __syncthreads();
    if (threadIdx.x < 32) {
        p = threadIdx.x < 8 ? ws[threadIdx.x] : red_identity<OP>();
        p = red_warp<OP>(p);
    }
    return p;
}

// ------------------------------------------------------------ element views
template <int ELEM> struct El;
template <> struct El<HEXCUDA_ELEM_I8> { using T = int8_t; static constexpr int kPerVec = 16; };
template <> struct El<HEXCUDA_ELEM_U8> { using T = uint8_t; static constexpr int kPerVec = 16; };
template <> struct El<HEXCUDA_ELEM_I16> { using T = int16_t; static constexpr int kPerVec = 8; };
template <> struct El<HEXCUDA_ELEM_I32> { using T = int32_t; static constexpr int kPerVec = 4; };

// One element (scalar path and 16-bit / 32-bit vectors).
template <int OP>
__device__ __forceinline__ void red_elem(RedPart &p, long long x, long long y, long long idx) {
    if constexpr (OP == HEXCUDA_RED_SUM64) {
        p.v += x;
    } else if constexpr (OP == HEXCUDA_RED_SUM || OP == HEXCUDA_RED_MEAN) {
        p.v = (uint32_t)((uint32_t)p.v + (uint32_t)x);
    } else if constexpr (OP == HEXCUDA_RED_SUMSQ) {
        p.v = (uint32_t)((uint32_t)p.v + (uint32_t)x * (uint32_t)x);
    } else if constexpr (OP == HEXCUDA_RED_SUMSQ_DIFF) {
        const uint32_t d = (uint32_t)(x - y);
        p.v = (uint32_t)((uint32_t)p.v + d * d);
    } else if constexpr (OP == HEXCUDA_RED_DOT) {
        p.v = (uint32_t)((uint32_t)p.v + (uint32_t)x * (uint32_t)y);
    } else if constexpr (OP == HEXCUDA_RED_L1) {
        p.v = (uint32_t)((uint32_t)p.v + (uint32_t)(x < 0 ? -x : x));
    } else if constexpr (OP == HEXCUDA_RED_ABSMAX) {
        const long long ax = x < 0 ? -x : x;
        if (ax > p.v) p.v = ax;
    } else if constexpr (red_min(OP)) {
        if (x < p.v) p = RedPart{x, idx};
    } else {
        if (x > p.v) p = RedPart{x, idx};
    }
}

// byte form: 4 packed int8 / uint8 of a (and b) -> the thread's accumulators
// (acc: the uint32 sum; m: packed per-byte extremes)
template <int ELEM, int OP>
__device__ __forceinline__ void red_word(uint32_t &acc, uint32_t &m, uint32_t wa, uint32_t wb) {
    constexpr bool S = ELEM == HEXCUDA_ELEM_I8;
    if constexpr (OP == HEXCUDA_RED_SUM || OP == HEXCUDA_RED_MEAN) {
        acc = S ? (uint32_t)__dp4a((int)wa, 0x01010101, (int)acc) : __dp4a(wa, 0x01010101u, acc);
    } else if constexpr (OP == HEXCUDA_RED_SUMSQ) {
        acc = S ? (uint32_t)__dp4a((int)wa, (int)wa, (int)acc) : __dp4a(wa, wa, acc);
    } else if constexpr (OP == HEXCUDA_RED_DOT) {
        acc = S ? (uint32_t)__dp4a((int)wa, (int)wb, (int)acc) : __dp4a(wa, wb, acc);
    } else if constexpr (OP == HEXCUDA_RED_SUMSQ_DIFF) {
        // sum (a - b)^2 = sum a^2 + sum b^2 - 2 sum a b, exact modulo 2^32
        uint32_t aa, bb, ab;
        if constexpr (S) {
            aa = (uint32_t)__dp4a((int)wa, (int)wa, 0);
            bb = (uint32_t)__dp4a((int)wb, (int)wb, 0);
            ab = (uint32_t)__dp4a((int)wa, (int)wb, 0);
        } else {
            aa = __dp4a(wa, wa, 0u);
            bb = __dp4a(wb, wb, 0u);
            ab = __dp4a(wa, wb, 0u);
        }
        acc += aa + bb - 2u * ab;
    } else if constexpr (OP == HEXCUDA_RED_L1) {
        acc = __dp4a(S ? __vabs4(wa) : wa, 0x01010101u, acc);
    } else if constexpr (OP == HEXCUDA_RED_ABSMAX) {
        m = __vmaxu4(m, S ? __vabs4(wa) : wa);
    } else if constexpr (red_min(OP)) {
        m = S ? __vmins4(m, wa) : __vminu4(m, wa);
    } else {
        m = S ? __vmaxs4(m, wa) : __vmaxu4(m, wa);
    }
}

// extreme of the 4 packed bytes of m, as a value
template <int ELEM, int OP>
__device__ __forceinline__ long long red_bytes(uint32_t m) {
    constexpr bool S = ELEM == HEXCUDA_ELEM_I8 && OP != HEXCUDA_RED_ABSMAX;
    uint32_t h = m >> 16;
    if constexpr (red_min(OP)) {
        m = S ? __vmins4(m, h) : __vminu4(m, h);
        m = S ? __vmins4(m, m >> 8) : __vminu4(m, m >> 8);
    } else {
        m = S ? __vmaxs4(m, h) : __vmaxu4(m, h);
        m = S ? __vmaxs4(m, m >> 8) : __vmaxu4(m, m >> 8);
    }
    return S ? (long long)(int8_t)(m & 0xFFu) : (long long)(m & 0xFFu);
}

template <int ELEM, int OP>
__device__ __forceinline__ uint32_t red_m_init() {
    if constexpr (OP == HEXCUDA_RED_ABSMAX) return 0u;
    else if constexpr (ELEM == HEXCUDA_ELEM_I8) return red_min(OP) ? 0x7F7F7F7Fu : 0x80808080u;
    else return red_min(OP) ? 0xFFFFFFFFu : 0u;
}

// --------------------------------------------------------- reduction kernel
// Grid-stride over 16-byte vectors (four in flight per thread for the byte
// sums and extremes), then the scalar tail; one partial per block.
template <int ELEM, int OP>
__global__ void __launch_bounds__(256) reduce_int_kernel(const void *__restrict__ a,
                                                         const void *__restrict__ b, int64_t n,
                                                         int vec, RedPart *__restrict__ part) {
    using T = typename El<ELEM>::T;
    constexpr int kPer = El<ELEM>::kPerVec;
    constexpr bool kBytes = ELEM == HEXCUDA_ELEM_I8 || ELEM == HEXCUDA_ELEM_U8;
    constexpr bool kS = ELEM == HEXCUDA_ELEM_I8;
    constexpr bool kB = red_needs_b(OP);
    const T *pa = reinterpret_cast<const T *>(a);
    const T *pb = reinterpret_cast<const T *>(b);
    const uint4 *va = reinterpret_cast<const uint4 *>(a);
    const uint4 *vb = reinterpret_cast<const uint4 *>(b);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // the one-block finalize launched after this kernel may start now (it
    // waits for this grid's partials before reading them)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    RedPart p = red_identity<OP>();
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n / kPer;
        if constexpr (kBytes && !red_arg(OP) && OP != HEXCUDA_RED_SUM64) {
            uint32_t acc = 0, m = red_m_init<ELEM, OP>();
            int64_t v = t;
            for (; v + 3 * stride < nv; v += 4 * stride) {
                uint4 xa[4], xb[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    xa[u] = __ldcs(va + v + u * stride);
                    xb[u] = kB ? __ldcs(vb + v + u * stride) : xa[u];
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    red_word<ELEM, OP>(acc, m, xa[u].x, xb[u].x);
                    red_word<ELEM, OP>(acc, m, xa[u].y, xb[u].y);
                    red_word<ELEM, OP>(acc, m, xa[u].z, xb[u].z);
                    red_word<ELEM, OP>(acc, m, xa[u].w, xb[u].w);
                }
            }
            for (; v < nv; v += stride) {
                const uint4 xa = __ldcs(va + v);
                const uint4 xb = kB ? __ldcs(vb + v) : xa;
                red_word<ELEM, OP>(acc, m, xa.x, xb.x);
                red_word<ELEM, OP>(acc, m, xa.y, xb.y);
                red_word<ELEM, OP>(acc, m, xa.z, xb.z);
                red_word<ELEM, OP>(acc, m, xa.w, xb.w);
            }
            if constexpr (red_ext(OP)) {
                if (t < nv) p.v = red_bytes<ELEM, OP>(m);
            } else {
                p.v = acc;
            }
        } else if constexpr (kBytes && red_arg(OP)) {
            // arg reductions: the vector's extreme, then its first byte only
            // when it improves on the thread's best
            for (int64_t v = t; v < nv; v += stride) {
                const uint4 x = __ldcs(va + v);
                uint32_t m;
                if constexpr (red_min(OP))
                    m = kS ? __vmins4(__vmins4(x.x, x.y), __vmins4(x.z, x.w))
                           : __vminu4(__vminu4(x.x, x.y), __vminu4(x.z, x.w));
                else
                    m = kS ? __vmaxs4(__vmaxs4(x.x, x.y), __vmaxs4(x.z, x.w))
                           : __vmaxu4(__vmaxu4(x.x, x.y), __vmaxu4(x.z, x.w));
                const long long cm = red_bytes<ELEM, OP>(m);
                if (red_min(OP) ? cm < p.v : cm > p.v) {
                    const uint32_t w[4] = {x.x, x.y, x.z, x.w};
                    int j = 0;
                    for (; j < 15; j++) {
                        const uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                        if ((kS ? (long long)(int8_t)byte : (long long)byte) == cm) break;
                    }
                    p = RedPart{cm, v * kPer + j};
                }
            }
        } else {
            for (int64_t v = t; v < nv; v += stride) {
                const uint4 x = __ldcs(va + v);
                const uint4 y = kB ? __ldcs(vb + v) : x;
                const T *ex = reinterpret_cast<const T *>(&x);
                const T *ey = reinterpret_cast<const T *>(&y);
#pragma unroll
                for (int e = 0; e < kPer; e++) red_elem<OP>(p, ex[e], ey[e], v * kPer + e);
            }
        }
        done = nv * kPer;
    }
    for (int64_t i = done + t; i < n; i += stride)
        red_elem<OP>(p, (long long)pa[i], kB ? (long long)pb[i] : 0ll, i);
    p = red_block<OP>(p);
    if (threadIdx.x == 0) part[blockIdx.x] = p;
}

// Combines the block partials; `one` gets the combined partial (indices
// offset by `base`), `out` the op's result.
template <int OP>
__global__ void __launch_bounds__(256) red_finalize_kernel(const RedPart *__restrict__ part,
                                                           int nparts, int64_t n, long long base,
                                                           RedPart *one, void *out) {
    // launched as a programmatic dependent of the block-partials kernel: wait
    // until that grid has finished and its partials are visible (a no-op when
    // launched without one)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    RedPart p = red_identity<OP>();
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) p = red_combine<OP>(p, part[i]);
    p = red_block<OP>(p);
    if (threadIdx.x == 0) {
        if constexpr (red_arg(OP)) p.i += base;
        if (one) *one = p;
        if (out) red_write<OP>(p, n, out);
    }
}

__host__ __device__ inline bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

template <int ELEM, int OP>
int reduce_launch(Dev *d, const void *a, const void *b, int64_t n, long long base, RedPart *one,
                  void *out) {
    constexpr int kPer = El<ELEM>::kPerVec;
    constexpr auto kern = reduce_int_kernel<ELEM, OP>;
    const int vec = al16(a) && (!red_needs_b(OP) || al16(b));
    const int64_t work = vec ? std::max<int64_t>(1, n / kPer / 4) : n;
    const int blocks = n > 0 ? resident_blocks<kern>(d, work) : 0;
    RedPart *part = reinterpret_cast<RedPart *>(
        scratch(d, kSlotRedPart, sizeof(RedPart) * (size_t)(blocks > 0 ? blocks : 1)));
    if (!part) return HEXCUDA_ERR_OOM;
    launch_begin(d);
    if (blocks > 0) kern<<<blocks, 256, 0, d->stream>>>(a, b, n, vec, part);
    if (blocks > 0 && vec) note_mech(kMechVec128);
    // the finalize as a programmatic dependent: its launch overlaps the
    // partials kernel's tail instead of following it
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = d->stream;
    cfg.attrs = attr;
    cfg.numAttrs = blocks > 0 ? 1 : 0;
    if (int rc = check(cudaLaunchKernelEx(&cfg, red_finalize_kernel<OP>, (const RedPart *)part,
                                          blocks, n, base, one, out),
                       "launch reduce finalize"))
        return rc;
    return launch_end(d, "reduce_int", blocks > 0 ? 2 : 1);
}

template <int ELEM>
int reduce_by_op(Dev *d, const void *a, const void *b, int64_t n, int op, long long base,
                 RedPart *one, void *out) {
    switch (op) {
#define HX_RED_OP(O) \
    case O:          \
        return reduce_launch<ELEM, O>(d, a, b, n, base, one, out);
        HX_RED_OP(HEXCUDA_RED_SUM)
        HX_RED_OP(HEXCUDA_RED_SUM64)
        HX_RED_OP(HEXCUDA_RED_SUMSQ)
        HX_RED_OP(HEXCUDA_RED_SUMSQ_DIFF)
        HX_RED_OP(HEXCUDA_RED_DOT)
        HX_RED_OP(HEXCUDA_RED_L1)
        HX_RED_OP(HEXCUDA_RED_ABSMAX)
        HX_RED_OP(HEXCUDA_RED_MAX)
        HX_RED_OP(HEXCUDA_RED_MIN)
        HX_RED_OP(HEXCUDA_RED_ARGMAX)
        HX_RED_OP(HEXCUDA_RED_ARGMIN)
        HX_RED_OP(HEXCUDA_RED_TOP1)
        HX_RED_OP(HEXCUDA_RED_MEAN)
#undef HX_RED_OP
    }
    return fail(HEXCUDA_ERR_ARG, "reduce_int: op %d", op);
}

int reduce_dispatch(Dev *d, const void *a, const void *b, int elem, int64_t n, int op,
                    long long base, RedPart *one, void *out) {
    switch (elem) {
        case HEXCUDA_ELEM_I8: return reduce_by_op<HEXCUDA_ELEM_I8>(d, a, b, n, op, base, one, out);
        case HEXCUDA_ELEM_U8: return reduce_by_op<HEXCUDA_ELEM_U8>(d, a, b, n, op, base, one, out);
        case HEXCUDA_ELEM_I16: return reduce_by_op<HEXCUDA_ELEM_I16>(d, a, b, n, op, base, one, out);
        case HEXCUDA_ELEM_I32: return reduce_by_op<HEXCUDA_ELEM_I32>(d, a, b, n, op, base, one, out);
    }
    return fail(HEXCUDA_ERR_ARG, "reduce_int: element type %d", elem);
}

int reduce_check(const char *name, const void *a, const void *b, int elem, int64_t n, int op,
                 const void *out) {
    if (elem < HEXCUDA_ELEM_I8 || elem > HEXCUDA_ELEM_I32 || op < HEXCUDA_RED_SUM ||
        op > HEXCUDA_RED_MEAN || n < 0)
        return fail(HEXCUDA_ERR_ARG, "%s: elem %d op %d n %lld", name, elem, op, (long long)n);
    if (n == 0 && (red_arg(op) || op == HEXCUDA_RED_MEAN))
        return fail(HEXCUDA_ERR_ARG, "%s: op %d needs n >= 1", name, op);
    if (!out || (n > 0 && (!a || (red_needs_b(op) && !b))))
        return fail(HEXCUDA_ERR_ARG, "%s: null pointer", name);
    return HEXCUDA_OK;
}

// host-side combination of per-device partials
template <int OP>
void red_host_finish(const RedPart *parts, int np, int64_t n, void *out) {
    RedPart p = red_identity<OP>();
    for (int k = 0; k < np; k++) p = red_combine<OP>(p, parts[k]);
    red_write<OP>(p, n, out);
}

void red_host_finish_op(int op, const RedPart *parts, int np, int64_t n, void *out) {
    switch (op) {
#define HX_RED_FIN(O) \
    case O:           \
        red_host_finish<O>(parts, np, n, out); break;
        HX_RED_FIN(HEXCUDA_RED_SUM)
        HX_RED_FIN(HEXCUDA_RED_SUM64)
        HX_RED_FIN(HEXCUDA_RED_SUMSQ)
        HX_RED_FIN(HEXCUDA_RED_SUMSQ_DIFF)
        HX_RED_FIN(HEXCUDA_RED_DOT)
        HX_RED_FIN(HEXCUDA_RED_L1)
        HX_RED_FIN(HEXCUDA_RED_ABSMAX)
        HX_RED_FIN(HEXCUDA_RED_MAX)
        HX_RED_FIN(HEXCUDA_RED_MIN)
        HX_RED_FIN(HEXCUDA_RED_ARGMAX)
        HX_RED_FIN(HEXCUDA_RED_ARGMIN)
        HX_RED_FIN(HEXCUDA_RED_TOP1)
        HX_RED_FIN(HEXCUDA_RED_MEAN)
#undef HX_RED_FIN
    }
}

// ------------------------------------------------------ elementwise max/min
template <int ELEM, bool MIN>
__device__ __forceinline__ uint32_t mm_word(uint32_t x, uint32_t y) {
    if constexpr (ELEM == HEXCUDA_ELEM_I8) return MIN ? __vmins4(x, y) : __vmaxs4(x, y);
    else if constexpr (ELEM == HEXCUDA_ELEM_U8) return MIN ? __vminu4(x, y) : __vmaxu4(x, y);
    else return MIN ? __vmins2(x, y) : __vmaxs2(x, y);
}

// out = max / min(a, b), or (a, c) when SCALAR; cw = c replicated per lane
template <int ELEM, bool MIN, bool SCALAR>
__global__ void __launch_bounds__(256) minmax_ew_kernel(const void *__restrict__ a,
                                                        const void *__restrict__ b, uint32_t cw,
                                                        int32_t c, void *__restrict__ out,
                                                        int64_t n, int vec) {
    using T = typename El<ELEM>::T;
    constexpr int kPer = El<ELEM>::kPerVec;
    const T *pa = reinterpret_cast<const T *>(a);
    const T *pb = reinterpret_cast<const T *>(b);
    T *po = reinterpret_cast<T *>(out);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n / kPer;
        const uint4 *va = reinterpret_cast<const uint4 *>(a);
        const uint4 *vb = reinterpret_cast<const uint4 *>(b);
        uint4 *vo = reinterpret_cast<uint4 *>(out);
        for (int64_t v = t; v < nv; v += stride) {
            const uint4 x = __ldcs(va + v);
            const uint4 y = SCALAR ? make_uint4(cw, cw, cw, cw) : __ldcs(vb + v);
            __stcs(vo + v, make_uint4(mm_word<ELEM, MIN>(x.x, y.x), mm_word<ELEM, MIN>(x.y, y.y),
                                      mm_word<ELEM, MIN>(x.z, y.z), mm_word<ELEM, MIN>(x.w, y.w)));
        }
        done = nv * kPer;
    }
    for (int64_t i = done + t; i < n; i += stride) {
        const T x = pa[i];
        const T y = SCALAR ? (T)c : pb[i];
        po[i] = MIN ? (x < y ? x : y) : (x > y ? x : y);
    }
}

template <int ELEM, bool MIN>
int minmax_launch(Dev *d, const void *a, const void *b, int32_t c, void *out, int64_t n) {
    constexpr int kPer = El<ELEM>::kPerVec;
    const bool scalar = b == nullptr;
    const int vec = al16(a) && al16(out) && (scalar || al16(b));
    const int64_t work = vec ? std::max<int64_t>(1, n / kPer) : n;
    uint32_t cw;
    if (ELEM == HEXCUDA_ELEM_I16) cw = ((uint32_t)c & 0xFFFFu) * 0x00010001u;
    else cw = ((uint32_t)c & 0xFFu) * 0x01010101u;
    launch_begin(d);
    if (scalar) {
        constexpr auto kern = minmax_ew_kernel<ELEM, MIN, true>;
        kern<<<resident_blocks<kern>(d, work), 256, 0, d->stream>>>(a, b, cw, c, out, n, vec);
    } else {
        constexpr auto kern = minmax_ew_kernel<ELEM, MIN, false>;
        kern<<<resident_blocks<kern>(d, work), 256, 0, d->stream>>>(a, b, cw, c, out, n, vec);
    }
    return launch_end(d, "minmax_ew");
}

// --------------------------------------------------------------- group sums
// w = 4 with 16-byte aligned operands: four outputs per 16-byte load (dp4a
// against ones), one 16-byte store.
// With b: out[k] = sum_j a[4k + j] b[4k + j] (hvx_vrmpy_i8_dot), dp4a against b.
template <bool DOT>
__global__ void __launch_bounds__(256) group_sum4_kernel(const int8_t *__restrict__ a,
                                                         const int8_t *__restrict__ b,
                                                         int32_t *__restrict__ out, int64_t g) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nv = g / 4;
    for (int64_t v = t; v < nv; v += stride) {
        const uint4 x = __ldcs(reinterpret_cast<const uint4 *>(a) + v);
        const uint4 y = DOT ? __ldcs(reinterpret_cast<const uint4 *>(b) + v)
                            : make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
        __stcs(reinterpret_cast<int4 *>(out) + v,
               make_int4(__dp4a((int)x.x, (int)y.x, 0), __dp4a((int)x.y, (int)y.y, 0),
                         __dp4a((int)x.z, (int)y.z, 0), __dp4a((int)x.w, (int)y.w, 0)));
    }
    for (int64_t k = nv * 4 + t; k < g; k += stride) {
        int32_t s = 0;
        for (int j = 0; j < 4; j++) s += (int32_t)a[4 * k + j] * (DOT ? (int32_t)b[4 * k + j] : 1);
        out[k] = s;
    }
}

template <bool DOT>
__global__ void __launch_bounds__(256) group_sum_kernel(const int8_t *__restrict__ a,
                                                        const int8_t *__restrict__ b,
                                                        int32_t *__restrict__ out, int64_t g,
                                                        int w) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < g; k += stride) {
        uint32_t s = 0;
        for (int j = 0; j < w; j++)
            s += (uint32_t)((int32_t)a[k * w + j] * (DOT ? (int32_t)b[k * w + j] : 1));
        out[k] = (int32_t)s;
    }
}

// ------------------------------------------------------------- prefix max
// Three passes, no block waits on another: (1) each 16 KB chunk's maximum,
// (2) one block turns those into each chunk's carry-in (the maximum of all
// earlier chunks, -128 for the first), (3) each chunk's inclusive scan with
// its carry-in.  Thread t of a block owns bytes [64 t, 64 t + 64) of the chunk.
constexpr int kScanPerThread = 64;
constexpr int kScanChunk = 256 * kScanPerThread;

__device__ __forceinline__ int scan_load(const int8_t *in, int64_t n, int64_t off, uint32_t (&w)[16]) {
    // 64 bytes from off (n bounds; bytes past the end read as -128)
    if (off + kScanPerThread <= n && al16(in + off)) {
        const uint4 *src = reinterpret_cast<const uint4 *>(in + off);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint4 x = __ldg(src + q);
            w[4 * q] = x.x, w[4 * q + 1] = x.y, w[4 * q + 2] = x.z, w[4 * q + 3] = x.w;
        }
        return kScanPerThread;
    }
#pragma unroll
    for (int k = 0; k < 16; k++) w[k] = 0x80808080u;
    int cnt = 0;
    for (int j = 0; j < kScanPerThread && off + j < n; j++, cnt++) {
        const uint32_t byte = (uint32_t)(uint8_t)in[off + j];
        w[j >> 2] = (w[j >> 2] & ~(0xFFu << (8 * (j & 3)))) | (byte << (8 * (j & 3)));
    }
    return cnt;
}

__device__ __forceinline__ int block_max_i32(int v) {
    __shared__ int ws[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_down_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < 8 ? ws[threadIdx.x] : -128;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) v = max(v, __shfl_down_sync(0xffffffffu, v, o));
    }
    return v;
}

// exclusive max-scan of one value per thread over the 256-thread block
__device__ __forceinline__ int block_excl_max(int v) {
    __shared__ int ws[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = max(incl, u);
    }
    if (lane == 31) ws[warp] = incl;
    __syncthreads();
    int before = -128;
    for (int k = 0; k < warp; k++) before = max(before, ws[k]);
    int excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = -128;
    return max(before, excl);
}

__global__ void __launch_bounds__(256) scan_chunk_max_kernel(const int8_t *__restrict__ in,
                                                             int64_t n, int *__restrict__ cmax) {
    uint32_t w[16];
    scan_load(in, n, (int64_t)blockIdx.x * kScanChunk + (int64_t)threadIdx.x * kScanPerThread, w);
    uint32_t m = 0x80808080u;
#pragma unroll
    for (int k = 0; k < 16; k++) m = __vmaxs4(m, w[k]);
    m = __vmaxs4(m, m >> 16);
    m = __vmaxs4(m, m >> 8);
    const int v = block_max_i32((int)(int8_t)(m & 0xFFu));
    if (threadIdx.x == 0) cmax[blockIdx.x] = v;
}

// one block: carry[c] = max(-128, cmax[0..c))
__global__ void __launch_bounds__(256) scan_carry_kernel(const int *__restrict__ cmax, int64_t nc,
                                                         int *__restrict__ carry) {
    const int64_t per = (nc + 255) / 256;
    const int64_t c0 = threadIdx.x * per, c1 = min(nc, c0 + per);
    int tot = -128;
    for (int64_t c = c0; c < c1; c++) tot = max(tot, cmax[c]);
    int run = block_excl_max(tot);
    for (int64_t c = c0; c < c1; c++) {
        carry[c] = run;
        run = max(run, cmax[c]);
    }
}

__global__ void __launch_bounds__(256) scan_apply_kernel(const int8_t *__restrict__ in,
                                                         int8_t *__restrict__ out, int64_t n,
                                                         const int *__restrict__ carry) {
    const int64_t off = (int64_t)blockIdx.x * kScanChunk + (int64_t)threadIdx.x * kScanPerThread;
    uint32_t w[16];
    const int cnt = scan_load(in, n, off, w);
    // thread-local inclusive prefix over its 64 bytes
    int run = -128;
#pragma unroll
    for (int j = 0; j < kScanPerThread; j++) {
        const int x = (int)(int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xFFu);
        run = max(run, x);
        w[j >> 2] = (w[j >> 2] & ~(0xFFu << (8 * (j & 3)))) | ((uint32_t)(uint8_t)run << (8 * (j & 3)));
    }
    const int cin = max(carry[blockIdx.x], block_excl_max(run));
    const uint32_t cw = ((uint32_t)(uint8_t)cin) * 0x01010101u;
#pragma unroll
    for (int k = 0; k < 16; k++) w[k] = __vmaxs4(w[k], cw);
    if (cnt == kScanPerThread && al16(out + off)) {
        uint4 *dst = reinterpret_cast<uint4 *>(out + off);
#pragma unroll
        for (int q = 0; q < 4; q++) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    } else {
        for (int j = 0; j < cnt; j++) out[off + j] = (int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xFFu);
    }
}

// ------------------------------------------------------- head-group reduce
// Y[g][i] = requant(sum of the HPG head planes of group g at i); 16 positions
// per thread step when MN % 16 == 0 and both planes are 16-byte aligned.
__global__ void __launch_bounds__(256) head_group_reduce_kernel(const int8_t *__restrict__ X,
                                                                int8_t *__restrict__ Y, int G,
                                                                int HPG, int64_t MN, int32_t mult,
                                                                int shift, int vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t nv = MN / 16, units = (int64_t)G * nv;
        for (int64_t u = t; u < units; u += stride) {
            const int64_t g = u / nv, v = u - g * nv;
            int32_t acc[16];
#pragma unroll
            for (int e = 0; e < 16; e++) acc[e] = 0;
            const uint4 *src = reinterpret_cast<const uint4 *>(X + g * HPG * MN) + v;
            for (int h = 0; h < HPG; h++) {
                const uint4 x = __ldcs(src + (int64_t)h * nv);
                const uint32_t q[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int e = 0; e < 16; e++) acc[e] += (int8_t)((q[e >> 2] >> (8 * (e & 3))) & 0xFFu);
            }
            uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
            for (int e = 0; e < 16; e++)
                o[e >> 2] |= ((uint32_t)requant_i8(acc[e], mult, shift, 0) & 0xFFu) << (8 * (e & 3));
            __stcs(reinterpret_cast<uint4 *>(Y + g * MN) + v, make_uint4(o[0], o[1], o[2], o[3]));
        }
    } else {
        const int64_t units = (int64_t)G * MN;
        for (int64_t u = t; u < units; u += stride) {
            const int64_t g = u / MN, i = u - g * MN;
            int32_t acc = 0;
            for (int h = 0; h < HPG; h++) acc += X[(g * HPG + h) * MN + i];
            Y[g * MN + i] = (int8_t)requant_i8(acc, mult, shift, 0);
        }
    }
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_reduce_int(int dev, const void *a, const void *b, int elem, int64_t n,
                                 int op, void *out) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (int rc = reduce_check("reduce_int", a, b, elem, n, op, out)) return rc;
    return reduce_dispatch(d, a, b, elem, n, op, 0, nullptr, out);
}

// Shards of the array over the devices; each device reduces its shard to one
// partial (arg indices already global), the host combines them.
HX_EXPORT int hexcuda_host_reduce_int(const void *a, const void *b, int elem, int64_t n, int op,
                                      void *out) {
    if (int rc = reduce_check("host_reduce_int", a, b, elem, n, op, out)) return rc;
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const size_t es = elem == HEXCUDA_ELEM_I32 ? 4 : (elem == HEXCUDA_ELEM_I16 ? 2 : 1);
    const int nd = ndev();
    std::vector<RedPart> host_parts(nd > 0 ? nd : 1);
    RedPart *pinned = reinterpret_cast<RedPart *>(host_parts.data());
    int np = 0, rc = HEXCUDA_OK;
    std::vector<int> used;
    scope_begin();
    for (int i = 0; i < nd && !rc; i++) {
        const int64_t r0 = n * i / nd, r1 = n * (i + 1) / nd;
        if (r1 <= r0 && !(n == 0 && i == 0)) continue;
        Dev *d = get_dev(i);
        if (!d) {
            rc = HEXCUDA_ERR_NODEV;
            break;
        }
        const int64_t nr = r1 - r0;
        // the host-entry staging slots (the two input operands)
        void *da = nr ? scratch(d, 8, (size_t)nr * es) : nullptr;
        void *db = nr && red_needs_b(op) ? scratch(d, 9, (size_t)nr * es) : nullptr;
        RedPart *one = reinterpret_cast<RedPart *>(scratch(d, kSlotRedOne, sizeof(RedPart)));
        if ((nr && !da) || (nr && red_needs_b(op) && !db) || !one) {
            rc = hexcuda_last_error();
            break;
        }
        if (nr)
            rc = check(cudaMemcpyAsync(da, reinterpret_cast<const uint8_t *>(a) + r0 * es, nr * es,
                                       cudaMemcpyHostToDevice, d->stream),
                       "h2d");
        if (!rc && db)
            rc = check(cudaMemcpyAsync(db, reinterpret_cast<const uint8_t *>(b) + r0 * es, nr * es,
                                       cudaMemcpyHostToDevice, d->stream),
                       "h2d");
        if (!rc) rc = reduce_dispatch(d, da, db, elem, nr, op, r0, one, nullptr);
        if (!rc)
            rc = check(cudaMemcpyAsync(pinned + np, one, sizeof(RedPart), cudaMemcpyDeviceToHost,
                                       d->stream),
                       "d2h");
        used.push_back(i);
        np++;
    }
    for (int i : used) {
        const int r = hexcuda_sync(i);
        if (r && !rc) rc = r;
    }
    scope_end();
    if (rc) return rc;
    red_host_finish_op(op, pinned, np, n, out);
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_minmax_ew(int dev, const void *a, const void *b, int32_t c, int elem, int op,
                                void *out, int64_t n) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0 || (op != 0 && op != 1) ||
        (elem != HEXCUDA_ELEM_I8 && elem != HEXCUDA_ELEM_U8 && elem != HEXCUDA_ELEM_I16))
        return fail(HEXCUDA_ERR_ARG, "minmax_ew: elem %d op %d n %lld", elem, op, (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (!a || !out) return fail(HEXCUDA_ERR_ARG, "minmax_ew: null pointer");
    if (elem == HEXCUDA_ELEM_I8)
        return op ? minmax_launch<HEXCUDA_ELEM_I8, true>(d, a, b, c, out, n)
                  : minmax_launch<HEXCUDA_ELEM_I8, false>(d, a, b, c, out, n);
    if (elem == HEXCUDA_ELEM_U8)
        return op ? minmax_launch<HEXCUDA_ELEM_U8, true>(d, a, b, c, out, n)
                  : minmax_launch<HEXCUDA_ELEM_U8, false>(d, a, b, c, out, n);
    return op ? minmax_launch<HEXCUDA_ELEM_I16, true>(d, a, b, c, out, n)
              : minmax_launch<HEXCUDA_ELEM_I16, false>(d, a, b, c, out, n);
}

namespace hx {
namespace {
template <bool DOT>
int group_launch(Dev *d, const int8_t *a, const int8_t *b, int32_t *out, int64_t g, int w) {
    launch_begin(d);
    if (w == 4 && al16(a) && al16(out) && (!DOT || al16(b))) {
        constexpr auto kern = group_sum4_kernel<DOT>;
        kern<<<resident_blocks<kern>(d, std::max<int64_t>(1, g / 4)), 256, 0, d->stream>>>(a, b, out, g);
    } else {
        constexpr auto kern = group_sum_kernel<DOT>;
        kern<<<resident_blocks<kern>(d, g), 256, 0, d->stream>>>(a, b, out, g, w);
    }
    return launch_end(d, DOT ? "group_dot_i8" : "group_sum_i8");
}
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_group_sum_i8(int dev, const int8_t *a, int32_t *out, int64_t g, int w) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (g < 0 || w < 1) return fail(HEXCUDA_ERR_ARG, "group_sum_i8: g %lld w %d", (long long)g, w);
    if (g == 0) return HEXCUDA_OK;
    if (!a || !out) return fail(HEXCUDA_ERR_ARG, "group_sum_i8: null pointer");
    return group_launch<false>(d, a, nullptr, out, g, w);
}

HX_EXPORT int hexcuda_group_dot_i8(int dev, const int8_t *a, const int8_t *b, int32_t *out,
                                   int64_t g, int w) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (g < 0 || w < 1) return fail(HEXCUDA_ERR_ARG, "group_dot_i8: g %lld w %d", (long long)g, w);
    if (g == 0) return HEXCUDA_OK;
    if (!a || !b || !out) return fail(HEXCUDA_ERR_ARG, "group_dot_i8: null pointer");
    return group_launch<true>(d, a, b, out, g, w);
}

HX_EXPORT int hexcuda_scan_max_i8(int dev, const int8_t *in, int8_t *out, int64_t n) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "scan_max_i8: n %lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (!in || !out) return fail(HEXCUDA_ERR_ARG, "scan_max_i8: null pointer");
    const int64_t nc = (n + kScanChunk - 1) / kScanChunk;
    if (nc > INT_MAX) return fail(HEXCUDA_ERR_ARG, "scan_max_i8: n %lld too large", (long long)n);
    int *cmax = reinterpret_cast<int *>(scratch(d, kSlotRedOne, sizeof(int) * (size_t)nc));
    int *carry = reinterpret_cast<int *>(scratch(d, kSlotScanCarry, sizeof(int) * (size_t)nc));
    if (!cmax || !carry) return HEXCUDA_ERR_OOM;
    launch_begin(d);
    scan_chunk_max_kernel<<<(unsigned)nc, 256, 0, d->stream>>>(in, n, cmax);
    scan_carry_kernel<<<1, 256, 0, d->stream>>>(cmax, nc, carry);
    scan_apply_kernel<<<(unsigned)nc, 256, 0, d->stream>>>(in, out, n, carry);
    return launch_end(d, "scan_max_i8", 3);
}

HX_EXPORT int hexcuda_head_group_reduce_i8(int dev, const int8_t *X, int8_t *Y, int H, int G,
                                           int64_t MN, int32_t mult, int shift) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (H < 0 || G < 1 || MN < 0 || shift < 0 || shift > 63)
        return fail(HEXCUDA_ERR_ARG, "head_group_reduce_i8: H %d G %d MN %lld shift %d", H, G,
                    (long long)MN, shift);
    if (MN == 0) return HEXCUDA_OK;
    if ((H / G > 0 && !X) || !Y) return fail(HEXCUDA_ERR_ARG, "head_group_reduce_i8: null pointer");
    const int HPG = H / G;
    const int vec = (MN % 16) == 0 && al16(X) && al16(Y);
    const int64_t work = vec ? (int64_t)G * (MN / 16) : (int64_t)G * MN;
    launch_begin(d);
    constexpr auto kern = head_group_reduce_kernel;
    kern<<<resident_blocks<kern>(d, work), 256, 0, d->stream>>>(X, Y, G, HPG, MN, mult, shift, vec);
    return launch_end(d, "head_group_reduce_i8");
}
