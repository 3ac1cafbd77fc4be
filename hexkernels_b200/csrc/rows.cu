// rows.cu -- HBM-bound row operators: softmax, layernorm, rmsnorm, row
// sum/max (fp32 and fp16 storage, fp32 arithmetic), and the single-row
// online-softmax update step.
//
// One 256-thread CTA owns one row.  When the row fits (C <= 256 * NV * E with
// E elements per 16-byte vector) and is 16-byte aligned, each thread loads NV
// 128-bit vectors once into registers (coalesced: consecutive threads read
// consecutive 16 B), the row statistics are reduced with warp shuffles plus
// one shared-memory exchange per statistic, and the output is written with
// 128-bit streaming stores: exactly one HBM read and one HBM write per
// element.  Rows that do not fit take a generic three-pass path whose later
// passes re-read the row from L2.
//
// Arithmetic follows the corpus's scalar references (cited per operator) in
// fp32: expf (not the fast approximation), IEEE division and sqrtf, and
// separately rounded multiply/add in the elementwise epilogues (__fmul_rn /
// __fadd_rn), so the only difference from the sequential reference is the
// order of the row sums.
#include <cuda_fp16.h>
#include <math.h>

#include "hx_internal.h"

namespace hx {
namespace {

constexpr int kNT = 256;            // threads per row CTA
constexpr int kWarps = kNT / 32;

template <typename T> struct VecT;
template <> struct VecT<float> {
    using V = float4;
    static constexpr int E = 4;
    __device__ static void unpack(const float4 &v, float *f) {
        f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    }
    __device__ static float4 pack(const float *f) { return make_float4(f[0], f[1], f[2], f[3]); }
    __device__ static float load1(const float *p) { return *p; }
    __device__ static void store1(float *p, float f) { *p = f; }
};
template <> struct VecT<__half> {
    using V = uint4;
    static constexpr int E = 8;
    __device__ static void unpack(const uint4 &v, float *f) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        for (int i = 0; i < 4; i++) {
            float2 t = __half22float2(h[i]);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
    __device__ static uint4 pack(const float *f) {
        uint4 v;
        __half2 *h = reinterpret_cast<__half2 *>(&v);
        for (int i = 0; i < 4; i++) h[i] = __halves2half2(__float2half_rn(f[2 * i]), __float2half_rn(f[2 * i + 1]));
        return v;
    }
    __device__ static float load1(const __half *p) { return __half2float(*p); }
    __device__ static void store1(__half *p, float f) { *p = __float2half_rn(f); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions; `sh` must hold kWarps floats and is used once.
__device__ __forceinline__ float block_sum(float v, float *sh) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; w++) r += sh[w];
    return r;
}
__device__ __forceinline__ float block_max(float v, float *sh) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = sh[0];
#pragma unroll
    for (int w = 1; w < kWarps; w++) r = fmaxf(r, sh[w]);
    return r;
}

template <typename V> __device__ __forceinline__ V ld_stream(const V *p) { return __ldcs(p); }
template <typename V> __device__ __forceinline__ void st_stream(V *p, const V &v) { __stcs(p, v); }

enum RowOp { kSoftmax = 0, kLayerNorm = 1, kRmsNorm = 2, kRowSum = 3, kRowMax = 4 };

// Register path: the row lives in registers, NV 16-byte vectors per thread.
template <typename T, int OP, int NV>
__global__ void __launch_bounds__(kNT) row_reg_kernel(const T *__restrict__ x,
                                                       const T *__restrict__ gamma,
                                                       const T *__restrict__ beta,
                                                       T *__restrict__ out,
                                                       float *__restrict__ red_out, int C,
                                                       float eps) {
    using VT = VecT<T>;
    using V = typename VT::V;
    constexpr int E = VT::E;
    __shared__ float sh0[kWarps], sh1[kWarps];
    const int row = blockIdx.x;
    const int nvec = C / E;
    const V *xr = reinterpret_cast<const V *>(x + (size_t)row * C);
    float f[NV][E];
#pragma unroll
    for (int k = 0; k < NV; k++) {
        int v = k * kNT + threadIdx.x;
        if (v < nvec) VT::unpack(ld_stream(xr + v), f[k]);
    }
    auto valid = [&](int k) { return k * kNT + (int)threadIdx.x < nvec; };

    if (OP == kSoftmax) {
        // fp16_softmax/reference.c:13-27: row max, expf(x - max), row sum, divide.
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k))
#pragma unroll
                for (int e = 0; e < E; e++) m = fmaxf(m, f[k][e]);
        m = block_max(m, sh0);
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k))
#pragma unroll
                for (int e = 0; e < E; e++) {
                    f[k][e] = expf(f[k][e] - m);
                    s += f[k][e];
                }
        s = block_sum(s, sh1);
        V *orow = reinterpret_cast<V *>(out + (size_t)row * C);
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k)) {
                float o[E];
#pragma unroll
                for (int e = 0; e < E; e++) o[e] = __fdiv_rn(f[k][e], s);
                st_stream(orow + k * kNT + threadIdx.x, VT::pack(o));
            }
    } else if (OP == kLayerNorm || OP == kRmsNorm) {
        // fp16_layernorm/reference.c:9-23 and fp16_rmsnorm/reference.c:7-16.
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k))
#pragma unroll
                for (int e = 0; e < E; e++) {
                    s1 += f[k][e];
                    s2 += f[k][e] * f[k][e];
                }
        float mean = 0.0f, inv;
        if (OP == kLayerNorm) {
            s1 = block_sum(s1, sh0);
            s2 = block_sum(s2, sh1);
            mean = __fdiv_rn(s1, (float)C);
            float var = __fsub_rn(__fdiv_rn(s2, (float)C), __fmul_rn(mean, mean));
            if (var < 0.0f) var = 0.0f;
            inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
        } else {
            s2 = block_sum(s2, sh1);
            inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(s2, (float)C), eps)));
        }
        const V *gv = reinterpret_cast<const V *>(gamma);
        const V *bv = reinterpret_cast<const V *>(beta);
        V *orow = reinterpret_cast<V *>(out + (size_t)row * C);
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k)) {
                int v = k * kNT + threadIdx.x;
                float g[E], b[E], o[E];
                VT::unpack(__ldg(gv + v), g);
                if (OP == kLayerNorm) VT::unpack(__ldg(bv + v), b);
#pragma unroll
                for (int e = 0; e < E; e++) {
                    if (OP == kLayerNorm) {
                        float d = __fmul_rn(__fsub_rn(f[k][e], mean), inv);
                        o[e] = __fadd_rn(__fmul_rn(d, g[e]), b[e]);
                    } else {
                        o[e] = __fmul_rn(__fmul_rn(f[k][e], inv), g[e]);
                    }
                }
                st_stream(orow + v, VT::pack(o));
            }
    } else {
        // kernels/mined/fp32_sum/reference.c:8-14 per row (sum), or row max.
        float r = (OP == kRowSum) ? 0.0f : -INFINITY;
#pragma unroll
        for (int k = 0; k < NV; k++)
            if (valid(k))
#pragma unroll
                for (int e = 0; e < E; e++) r = (OP == kRowSum) ? r + f[k][e] : fmaxf(r, f[k][e]);
        r = (OP == kRowSum) ? block_sum(r, sh0) : block_max(r, sh0);
        if (threadIdx.x == 0) red_out[row] = r;
    }
}

// Generic path: any C, any alignment; statistics in passes over global memory.
template <typename T, int OP>
__global__ void __launch_bounds__(kNT) row_generic_kernel(const T *__restrict__ x,
                                                           const T *__restrict__ gamma,
                                                           const T *__restrict__ beta,
                                                           T *__restrict__ out,
                                                           float *__restrict__ red_out, int C,
                                                           float eps) {
    using VT = VecT<T>;
    __shared__ float sh0[kWarps], sh1[kWarps];
    const int row = blockIdx.x;
    const T *xr = x + (size_t)row * C;
    T *orow = out ? out + (size_t)row * C : nullptr;
    if (OP == kSoftmax) {
        float m = -INFINITY;
        for (int j = threadIdx.x; j < C; j += kNT) m = fmaxf(m, VT::load1(xr + j));
        m = block_max(m, sh0);
        float s = 0.0f;
        for (int j = threadIdx.x; j < C; j += kNT) s += expf(VT::load1(xr + j) - m);
        s = block_sum(s, sh1);
        for (int j = threadIdx.x; j < C; j += kNT)
            VT::store1(orow + j, __fdiv_rn(expf(VT::load1(xr + j) - m), s));
    } else if (OP == kLayerNorm || OP == kRmsNorm) {
        float s1 = 0.0f, s2 = 0.0f;
        for (int j = threadIdx.x; j < C; j += kNT) {
            float v = VT::load1(xr + j);
            s1 += v;
            s2 += v * v;
        }
        float mean = 0.0f, inv;
        if (OP == kLayerNorm) {
            s1 = block_sum(s1, sh0);
            s2 = block_sum(s2, sh1);
            mean = __fdiv_rn(s1, (float)C);
            float var = __fsub_rn(__fdiv_rn(s2, (float)C), __fmul_rn(mean, mean));
            if (var < 0.0f) var = 0.0f;
            inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
        } else {
            s2 = block_sum(s2, sh1);
            inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(s2, (float)C), eps)));
        }
        for (int j = threadIdx.x; j < C; j += kNT) {
            float v = VT::load1(xr + j), g = VT::load1(gamma + j), o;
            if (OP == kLayerNorm)
                o = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), inv), g), VT::load1(beta + j));
            else
                o = __fmul_rn(__fmul_rn(v, inv), g);
            VT::store1(orow + j, o);
        }
    } else {
        float r = (OP == kRowSum) ? 0.0f : -INFINITY;
        for (int j = threadIdx.x; j < C; j += kNT) {
            float v = VT::load1(xr + j);
            r = (OP == kRowSum) ? r + v : fmaxf(r, v);
        }
        r = (OP == kRowSum) ? block_sum(r, sh0) : block_max(r, sh0);
        if (threadIdx.x == 0) red_out[row] = r;
    }
}

// RMS norm with one gain per row (rmsnorm_gain_fp16/reference.c:6-19):
// inv = 1 / sqrt(sum x^2 / C + eps), out = (fp16)((x inv) gain[row]).
__global__ void __launch_bounds__(kNT) rmsnorm_gain_f16_kernel(const __half *__restrict__ x,
                                                               const __half *__restrict__ gain,
                                                               __half *__restrict__ out, int C,
                                                               float eps) {
    __shared__ float sh[kWarps];
    const int row = blockIdx.x;
    const __half *xr = x + (size_t)row * C;
    float s2 = 0.0f;
    for (int j = threadIdx.x; j < C; j += kNT) {
        const float v = __half2float(xr[j]);
        s2 += v * v;
    }
    s2 = block_sum(s2, sh);
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(s2, (float)C), eps)));
    const float g = __half2float(gain[row]);
    __half *orow = out + (size_t)row * C;
    for (int j = threadIdx.x; j < C; j += kNT)
        orow[j] = __float2half_rn(__fmul_rn(__fmul_rn(__half2float(xr[j]), inv), g));
}

template <typename T, int OP, int NV>
void launch_reg(Dev *d, const T *x, const T *g, const T *b, T *o, float *ro, int R, int C,
                float eps) {
    row_reg_kernel<T, OP, NV><<<R, kNT, 0, d->stream>>>(x, g, b, o, ro, C, eps);
}

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

template <typename T, int OP>
int launch_rows(int dev, const T *x, const T *gamma, const T *beta, T *out, float *red_out,
                int R, int C, float eps, const char *name) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "%s: bad shape R=%d C=%d", name, R, C);
    if (R == 0) return HEXCUDA_OK;
    if (!x || ((OP <= kRmsNorm) && !out) || (OP > kRmsNorm && !red_out))
        return fail(HEXCUDA_ERR_ARG, "%s: null pointer", name);
    if ((OP == kLayerNorm || OP == kRmsNorm) && !gamma)
        return fail(HEXCUDA_ERR_ARG, "%s: null gamma", name);
    if (OP == kLayerNorm && !beta) return fail(HEXCUDA_ERR_ARG, "%s: null beta", name);
    constexpr int E = VecT<T>::E;
    const bool vec = (C % E == 0) && aligned16(x) && (!out || aligned16(out)) &&
                     (!gamma || aligned16(gamma)) && (!beta || aligned16(beta));
    const int nvec = C / E;
    launch_begin(d);
    if (vec && nvec <= kNT * 1)
        launch_reg<T, OP, 1>(d, x, gamma, beta, out, red_out, R, C, eps);
    else if (vec && nvec <= kNT * 2)
        launch_reg<T, OP, 2>(d, x, gamma, beta, out, red_out, R, C, eps);
    else if (vec && nvec <= kNT * 4)
        launch_reg<T, OP, 4>(d, x, gamma, beta, out, red_out, R, C, eps);
    else if (vec && nvec <= kNT * 8)
        launch_reg<T, OP, 8>(d, x, gamma, beta, out, red_out, R, C, eps);
    else
        row_generic_kernel<T, OP><<<R, kNT, 0, d->stream>>>(x, gamma, beta, out, red_out, C, eps);
    if (vec && nvec <= kNT * 8) note_mech(kMechVec128);
    return launch_end(d, name);
}

// online_softmax_step_fp16/reference.c:9-37 for one query row: a single CTA.
// p[] lives in dynamic shared memory (BLK floats); each thread owns output
// dimensions d and sums over j in the reference's order.
__global__ void __launch_bounds__(kNT) online_softmax_step_kernel(
    const __half *__restrict__ scores, const __half *__restrict__ V, __half *running_max,
    __half *running_sum, __half *acc, int BLK, int D) {
    extern __shared__ float p[];
    __shared__ float sh0[kWarps], sh1[kWarps];
    __shared__ float s_corr, s_mnew;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < BLK; j += kNT) m = fmaxf(m, __half2float(scores[j]));
    m = block_max(m, sh0);
    float m_old = __half2float(*running_max);
    float m_new = (m_old > m) ? m_old : m;
    float psum_part = 0.0f;
    for (int j = threadIdx.x; j < BLK; j += kNT) {
        float e = expf(__half2float(scores[j]) - m_new);
        p[j] = e;
        psum_part += e;
    }
    __syncthreads();
    // the reference sums p[j] sequentially; one thread does the same
    if (threadIdx.x == 0) {
        float ps = 0.0f;
        for (int j = 0; j < BLK; j++) ps += p[j];
        float corr = expf(m_old - m_new);
        s_corr = corr;
        s_mnew = m_new;
        sh1[0] = __fadd_rn(__fmul_rn(__half2float(*running_sum), corr), ps);
    }
    (void)psum_part;
    __syncthreads();
    float corr = s_corr;
    for (int dd = threadIdx.x; dd < D; dd += kNT) {
        float a = __fmul_rn(__half2float(acc[dd]), corr);
        for (int j = 0; j < BLK; j++) a = __fadd_rn(a, __fmul_rn(p[j], __half2float(V[(size_t)j * D + dd])));
        acc[dd] = __float2half_rn(a);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *running_max = __float2half_rn(s_mnew);
        *running_sum = __float2half_rn(sh1[0]);
    }
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_softmax_f32(int dev, const float *x, float *out, int R, int C) {
    return launch_rows<float, kSoftmax>(dev, x, nullptr, nullptr, out, nullptr, R, C, 0.f,
                                        "softmax_f32");
}
HX_EXPORT int hexcuda_softmax_f16(int dev, const uint16_t *x, uint16_t *out, int R, int C) {
    return launch_rows<__half, kSoftmax>(dev, (const __half *)x, nullptr, nullptr, (__half *)out,
                                         nullptr, R, C, 0.f, "softmax_f16");
}
HX_EXPORT int hexcuda_layernorm_f32(int dev, const float *x, const float *gamma,
                                    const float *beta, float *out, int R, int C, float eps) {
    return launch_rows<float, kLayerNorm>(dev, x, gamma, beta, out, nullptr, R, C, eps,
                                          "layernorm_f32");
}
HX_EXPORT int hexcuda_layernorm_f16(int dev, const uint16_t *x, const uint16_t *gamma,
                                    const uint16_t *beta, uint16_t *out, int R, int C,
                                    float eps) {
    return launch_rows<__half, kLayerNorm>(dev, (const __half *)x, (const __half *)gamma,
                                           (const __half *)beta, (__half *)out, nullptr, R, C,
                                           eps, "layernorm_f16");
}
HX_EXPORT int hexcuda_rmsnorm_f32(int dev, const float *x, const float *gamma, float *out,
                                  int R, int C, float eps) {
    return launch_rows<float, kRmsNorm>(dev, x, gamma, nullptr, out, nullptr, R, C, eps,
                                        "rmsnorm_f32");
}
HX_EXPORT int hexcuda_rmsnorm_f16(int dev, const uint16_t *x, const uint16_t *gamma,
                                  uint16_t *out, int R, int C, float eps) {
    return launch_rows<__half, kRmsNorm>(dev, (const __half *)x, (const __half *)gamma, nullptr,
                                         (__half *)out, nullptr, R, C, eps, "rmsnorm_f16");
}
HX_EXPORT int hexcuda_rmsnorm_gain_f16(int dev, const uint16_t *x, const uint16_t *gain,
                                       uint16_t *out, int R, int C, float eps) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "rmsnorm_gain_f16: R=%d C=%d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (!x || !gain || !out) return fail(HEXCUDA_ERR_ARG, "rmsnorm_gain_f16: null pointer");
    launch_begin(d);
    rmsnorm_gain_f16_kernel<<<R, kNT, 0, d->stream>>>((const __half *)x, (const __half *)gain,
                                                      (__half *)out, C, eps);
    return launch_end(d, "rmsnorm_gain_f16");
}
HX_EXPORT int hexcuda_rowreduce_f32(int dev, const float *x, float *out, int R, int C, int op) {
    if (op == 0)
        return launch_rows<float, kRowSum>(dev, x, nullptr, nullptr, nullptr, out, R, C, 0.f,
                                           "rowsum_f32");
    if (op == 1)
        return launch_rows<float, kRowMax>(dev, x, nullptr, nullptr, nullptr, out, R, C, 0.f,
                                           "rowmax_f32");
    return fail(HEXCUDA_ERR_ARG, "rowreduce_f32: op %d is not 0 (sum) or 1 (max)", op);
}

HX_EXPORT int hexcuda_online_softmax_step_f16(int dev, const uint16_t *scores, const uint16_t *V,
                                              uint16_t *running_max, uint16_t *running_sum,
                                              uint16_t *acc, int BLK, int D) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (BLK <= 0 || D < 0 || BLK > 48 * 1024)
        return fail(HEXCUDA_ERR_ARG, "online_softmax_step: BLK=%d D=%d (1 <= BLK <= 49152)", BLK, D);
    if (!scores || !V || !running_max || !running_sum || (D > 0 && !acc))
        return fail(HEXCUDA_ERR_ARG, "online_softmax_step: null pointer");
    size_t smem = sizeof(float) * (size_t)BLK;
    if (smem > 48 * 1024) {
        if (int rc = check(cudaFuncSetAttribute(online_softmax_step_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)smem),
                           "cudaFuncSetAttribute"))
            return rc;
    }
    launch_begin(d);
    online_softmax_step_kernel<<<1, kNT, smem, d->stream>>>(
        (const __half *)scores, (const __half *)V, (__half *)running_max, (__half *)running_sum,
        (__half *)acc, BLK, D);
    return launch_end(d, "online_softmax_step_f16");
}
