// cache_rope.cu -- the two position-indexed neighbours of the attention
// blocks:
//
//   kv_cache_update_i8   write one new int8 K row and V row per head into the
//                        caches at position pos (kernels/expert/
//                        kv_cache_update/reference.c:14-25): a scatter of
//                        heads x head_dim bytes into [heads][cache_len][head_dim]
//   rope_pair_f16        rotary embedding of interleaved fp16 pairs with one
//                        cos / sin per pair, in fp32 without contraction
//                        (rope_pair_fp16/reference.c:5-13), so the result is
//                        the reference's rounding for rounding
//
// Both are HBM-bound byte movers: 16-byte vectors where the rows allow them,
// grids sized by occupancy.
#include <cuda_fp16.h>

#include "ew_launch.cuh"
#include "hx_internal.h"

namespace hx {
namespace {

// one thread per 16-byte chunk of a head's row (VEC) or per byte
template <bool VEC>
__global__ void __launch_bounds__(256) kv_cache_update_kernel(
    int8_t *__restrict__ kc, int8_t *__restrict__ vc, const int8_t *__restrict__ kn,
    const int8_t *__restrict__ vn, int pos, int heads, int cache_len, int head_dim) {
    const int per = VEC ? head_dim / 16 : head_dim;
    const int64_t n = (int64_t)heads * per;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride) {
        const int h = (int)(t / per), c = (int)(t % per);
        const int64_t dst = ((int64_t)h * cache_len + pos) * head_dim;
        const int64_t src = (int64_t)h * head_dim;
        if constexpr (VEC) {
            reinterpret_cast<uint4 *>(kc + dst)[c] = reinterpret_cast<const uint4 *>(kn + src)[c];
            reinterpret_cast<uint4 *>(vc + dst)[c] = reinterpret_cast<const uint4 *>(vn + src)[c];
        } else {
            kc[dst + c] = kn[src + c];
            vc[dst + c] = vn[src + c];
        }
    }
}

// out[2p] = x[2p] c - x[2p+1] s, out[2p+1] = x[2p] s + x[2p+1] c, each
// product and sum rounded to fp32 separately (no fused multiply-add)
__global__ void __launch_bounds__(256) rope_pair_f16_kernel(const __half2 *__restrict__ x,
                                                            const __half *__restrict__ cs,
                                                            const __half *__restrict__ sn,
                                                            __half2 *__restrict__ out, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += stride) {
        const float2 v = __half22float2(x[p]);
        const float c = __half2float(cs[p]), s = __half2float(sn[p]);
        const float re = __fsub_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, s));
        const float im = __fadd_rn(__fmul_rn(v.x, s), __fmul_rn(v.y, c));
        out[p] = __halves2half2(__float2half_rn(re), __float2half_rn(im));
    }
}

inline bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_kv_cache_update_i8(int dev, int8_t *k_cache, int8_t *v_cache,
                                         const int8_t *k_new, const int8_t *v_new, int pos,
                                         int heads, int cache_len, int head_dim) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (heads < 0 || cache_len < 1 || head_dim < 0 || pos < 0 || pos >= cache_len)
        return fail(HEXCUDA_ERR_ARG, "kv_cache_update_i8: pos %d heads %d cache_len %d head_dim %d",
                    pos, heads, cache_len, head_dim);
    if (heads == 0 || head_dim == 0) return HEXCUDA_OK;
    if (!k_cache || !v_cache || !k_new || !v_new)
        return fail(HEXCUDA_ERR_ARG, "kv_cache_update_i8: null pointer");
    launch_begin(d);
    if (head_dim % 16 == 0 && al16(k_cache) && al16(v_cache) && al16(k_new) && al16(v_new)) {
        constexpr auto kern = kv_cache_update_kernel<true>;
        kern<<<resident_blocks<kern>(d, (int64_t)heads * (head_dim / 16)), 256, 0, d->stream>>>(
            k_cache, v_cache, k_new, v_new, pos, heads, cache_len, head_dim);
    } else {
        constexpr auto kern = kv_cache_update_kernel<false>;
        kern<<<resident_blocks<kern>(d, (int64_t)heads * head_dim), 256, 0, d->stream>>>(
            k_cache, v_cache, k_new, v_new, pos, heads, cache_len, head_dim);
    }
    return launch_end(d, "kv_cache_update_i8");
}

HX_EXPORT int hexcuda_rope_pair_f16(int dev, const uint16_t *x, const uint16_t *cos_t,
                                    const uint16_t *sin_t, uint16_t *out, int64_t n_pairs) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (n_pairs < 0) return fail(HEXCUDA_ERR_ARG, "rope_pair_f16: n_pairs %lld", (long long)n_pairs);
    if (n_pairs == 0) return HEXCUDA_OK;
    if (!x || !cos_t || !sin_t || !out) return fail(HEXCUDA_ERR_ARG, "rope_pair_f16: null pointer");
    if (((uintptr_t)x | (uintptr_t)out) & 3u)
        return fail(HEXCUDA_ERR_ARG, "rope_pair_f16: x and out must be 4-byte aligned");
    launch_begin(d);
    constexpr auto kern = rope_pair_f16_kernel;
    kern<<<resident_blocks<kern>(d, n_pairs), 256, 0, d->stream>>>(
        reinterpret_cast<const __half2 *>(x), reinterpret_cast<const __half *>(cos_t),
        reinterpret_cast<const __half *>(sin_t), reinterpret_cast<__half2 *>(out), n_pairs);
    return launch_end(d, "rope_pair_f16");
}
