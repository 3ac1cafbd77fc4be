// attn.cu -- fp16 scaled-dot-product attention with fp32 softmax statistics.
//
// O[h, i, :] = sum_j softmax_j(scale * Q[h,i,:] . K[h,j,:]) V[h, j, :], the
// keys j restricted to j <= i when causal.  Flash recurrence of
// kernels/expert/fp16_flash_attention_tile/kernel_api.h:12-27: running max m,
// running sum l and running output acc per query row, rescaled by
// exp(m_old - m_new) whenever the max grows; one division by l at the end.
//
// This file holds the CUDA-core path (any SQ, SK, D <= 256): one warp per
// query row, key/value tiles of 32 rows staged in shared memory as fp32 and
// shared by the CTA's 4 warps (4 consecutive query rows).  Lane t scores key
// t of the tile, the warp reduces the tile max/sum with shuffles, and lane t
// accumulates output dimensions t, t+32, ...
#include <cuda_fp16.h>
#include <math.h>

#include "hx_internal.h"

namespace hx {
namespace {

constexpr int kTileK = 32;
constexpr int kWarpsPerCta = 4;
constexpr int kMaxD = 256;

__global__ void __launch_bounds__(32 * kWarpsPerCta) attn_simt_kernel(
    const __half *__restrict__ Q, const __half *__restrict__ K, const __half *__restrict__ V,
    __half *__restrict__ O, int SQ, int SK, int D, float scale, int causal) {
    extern __shared__ float sm[];
    float *sK = sm;                         // [kTileK][D + 1]
    float *sV = sK + kTileK * (D + 1);      // [kTileK][D]
    float *sQ = sV + kTileK * D;            // [kWarpsPerCta][D]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int q0 = blockIdx.x * kWarpsPerCta;
    const int i = q0 + warp;
    const __half *Qh = Q + (size_t)h * SQ * D;
    const __half *Kh = K + (size_t)h * SK * D;
    const __half *Vh = V + (size_t)h * SK * D;
    if (i < SQ)
        for (int d = lane; d < D; d += 32) sQ[warp * D + d] = __half2float(Qh[(size_t)i * D + d]);
    constexpr int kPer = kMaxD / 32;
    float acc[kPer];
#pragma unroll
    for (int u = 0; u < kPer; u++) acc[u] = 0.0f;
    float m = -INFINITY, l = 0.0f;
    // keys visible to the last row of this CTA bound the loop for all warps
    int kend = SK;
    if (causal) kend = min(SK, q0 + kWarpsPerCta);
    for (int j0 = 0; j0 < kend; j0 += kTileK) {
        __syncthreads();
        for (int e = threadIdx.x; e < kTileK * D; e += blockDim.x) {
            int jj = e / D, d = e % D, j = j0 + jj;
            float kv = 0.0f, vv = 0.0f;
            if (j < SK) {
                kv = __half2float(Kh[(size_t)j * D + d]);
                vv = __half2float(Vh[(size_t)j * D + d]);
            }
            sK[jj * (D + 1) + d] = kv;
            sV[jj * D + d] = vv;
        }
        __syncthreads();
        if (i >= SQ) continue;
        const int j = j0 + lane;
        const bool vis = j < SK && (!causal || j <= i);
        float s = -INFINITY;
        if (vis) {
            float a = 0.0f;
            for (int d = 0; d < D; d++) a += sQ[warp * D + d] * sK[lane * (D + 1) + d];
            s = a * scale;
        }
        float tmax = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        if (tmax == -INFINITY) continue;   // no visible key in this tile
        const float m_new = fmaxf(m, tmax);
        const float corr = expf(m - m_new);   // 0 on the first visible tile
        const float p = vis ? expf(s - m_new) : 0.0f;
        float psum = p;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l = l * corr + psum;
#pragma unroll
        for (int u = 0; u < kPer; u++) acc[u] *= corr;
        for (int jj = 0; jj < kTileK; jj++) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
#pragma unroll
            for (int u = 0; u < kPer; u++) {
                const int d = lane + 32 * u;
                if (d < D) acc[u] += pj * sV[jj * D + d];
            }
        }
        m = m_new;
    }
    if (i < SQ) {
        __half *Oh = O + (size_t)h * SQ * D + (size_t)i * D;
#pragma unroll
        for (int u = 0; u < kPer; u++) {
            const int d = lane + 32 * u;
            if (d < D) Oh[d] = __float2half_rn(l > 0.0f ? acc[u] / l : 0.0f);
        }
    }
}

}  // namespace

int attn_tc_launch(Dev *d, const __half *Q, const __half *K, const __half *V, __half *O, int BH,
                   int SQ, int SK, int D, float scale, int causal, bool *handled);

}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_attn_f16(int dev, const uint16_t *Q, const uint16_t *K, const uint16_t *V,
                               uint16_t *O, int BH, int SQ, int SK, int D, float scale,
                               int causal) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (BH < 0 || SQ < 0 || SK <= 0 || D <= 0 || D > kMaxD)
        return fail(HEXCUDA_ERR_ARG, "attn_f16: BH=%d SQ=%d SK=%d D=%d (1 <= D <= %d)", BH, SQ, SK,
                    D, kMaxD);
    if (BH == 0 || SQ == 0) return HEXCUDA_OK;
    if (!Q || !K || !V || !O) return fail(HEXCUDA_ERR_ARG, "attn_f16: null pointer");
    if (BH > 65535) return fail(HEXCUDA_ERR_ARG, "attn_f16: BH=%d > 65535", BH);
    launch_begin(d);
    bool handled = false;
    int rc = attn_tc_launch(d, (const __half *)Q, (const __half *)K, (const __half *)V,
                            (__half *)O, BH, SQ, SK, D, scale, causal, &handled);
    if (rc) return rc;
    if (!handled) {
        size_t smem = sizeof(float) * ((size_t)kTileK * (D + 1) + (size_t)kTileK * D +
                                       (size_t)kWarpsPerCta * D);
        if (smem > 48 * 1024) {
            if (int r = check(cudaFuncSetAttribute(attn_simt_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem),
                              "cudaFuncSetAttribute(attn)"))
                return r;
        }
        dim3 grid((unsigned)((SQ + kWarpsPerCta - 1) / kWarpsPerCta), (unsigned)BH);
        attn_simt_kernel<<<grid, 32 * kWarpsPerCta, smem, d->stream>>>(
            (const __half *)Q, (const __half *)K, (const __half *)V, (__half *)O, SQ, SK, D, scale,
            causal);
    }
    return launch_end(d, "attn_f16");
}
