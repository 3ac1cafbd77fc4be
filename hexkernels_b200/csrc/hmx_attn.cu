// hmx_attn.cu -- the HMX-convention fused QK^T -> AV block
// (kernels/expert/i8_attention_qkt_av_hmx/reference.c):
//
//     Sc[i][j]  = sx12((sum_d Q[i][d] K[j][d] * 17 + 8) >> 4)      (int, 12-bit)
//     out[i][d] = sx12((sum_j Sc[i][j] V[j][d] * 17 + 8) >> 4)     (int32)
//
// on the tcgen05 u8 x s8 engine.  The second product's left operand is a
// signed 12-bit value, not u8, so it is split exactly into bytes:
// Sc = 256 hi + lo with lo = Sc & 0xFF (u8) and hi = Sc >> 8 in [-8, 7],
// carried as hi + 8 (u8) with the engine's zero point 8.  Then
//     sum_j Sc V = 256 (sum_j (hi+8 - 8) V) + sum_j lo V
// and the two accumulators (the engine's raw int32 store) are combined with
// the reference's int32 wrap-around arithmetic before the final field.
#include "hx_internal.h"

namespace hx {
namespace {

constexpr int kSlotSc = 3, kSlotLo = 4, kSlotHi = 5, kSlotAccLo = 6, kSlotAccHi = 7;

__global__ void __launch_bounds__(256) split_bytes_kernel(const int32_t *__restrict__ sc,
                                                          uint8_t *__restrict__ lo,
                                                          uint8_t *__restrict__ hi, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t v = sc[i];          // in [-2048, 2047]
        lo[i] = (uint8_t)(v & 0xFF);
        hi[i] = (uint8_t)((v >> 8) + 8);
    }
}

__global__ void __launch_bounds__(256) combine_field_kernel(const int32_t *__restrict__ acc_hi,
                                                            const int32_t *__restrict__ acc_lo,
                                                            int32_t *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t acc = ((uint32_t)acc_hi[i] << 8) + (uint32_t)acc_lo[i];
        const int32_t f = (int32_t)(acc * 17u + 8u) >> 4;
        out[i] = (int32_t)((uint32_t)f << 20) >> 20;
    }
}

unsigned grid_for(const Dev *d, int64_t n) {
    int64_t b = (n + 255) / 256;
    const int64_t cap = (int64_t)d->sms * 8;
    return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_attn_qkt_av_hmx(int dev, const uint8_t *Q, const int8_t *K, const int8_t *V,
                                      int32_t *out, int SQ, int SK, int D) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (SQ < 0 || SK < 0 || D < 0)
        return fail(HEXCUDA_ERR_ARG, "attn_qkt_av_hmx: SQ=%d SK=%d D=%d", SQ, SK, D);
    if (SQ == 0 || D == 0) return HEXCUDA_OK;
    if (!Q || !K || !V || !out) return fail(HEXCUDA_ERR_ARG, "attn_qkt_av_hmx: null pointer");
    const int64_t ss = (int64_t)SQ * SK, sd = (int64_t)SQ * D;
    int32_t *sc = reinterpret_cast<int32_t *>(scratch(d, kSlotSc, (size_t)ss * 4));
    uint8_t *lo = reinterpret_cast<uint8_t *>(scratch(d, kSlotLo, (size_t)ss));
    uint8_t *hi = reinterpret_cast<uint8_t *>(scratch(d, kSlotHi, (size_t)ss));
    int32_t *alo = reinterpret_cast<int32_t *>(scratch(d, kSlotAccLo, (size_t)sd * 4));
    int32_t *ahi = reinterpret_cast<int32_t *>(scratch(d, kSlotAccHi, (size_t)sd * 4));
    if (!sc || !lo || !hi || !alo || !ahi) return HEXCUDA_ERR_OOM;
    // Sc = sx12 field of Q K^T (K is [S, D]: the K-major operand)
    if (int rc = hexcuda_gemm_hmx_ex(dev, Q, K, 1, nullptr, nullptr, HEXCUDA_HMX_RES_NONE, nullptr, sc,
                                     HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 0, SQ, SK, D, 0))
        return rc;
    launch_begin(d);
    split_bytes_kernel<<<grid_for(d, ss), 256, 0, d->stream>>>(sc, lo, hi, ss);
    if (int rc = launch_end(d, "attn_qkt_av_hmx split")) return rc;
    if (int rc = hexcuda_gemm_hmx_ex(dev, lo, V, 0, nullptr, nullptr, HEXCUDA_HMX_RES_NONE, nullptr, alo,
                                     HEXCUDA_HMX_STORE_ACC_I32, HEXCUDA_HMX_ACT_NONE, 0, SQ, D, SK, 0))
        return rc;
    if (int rc = hexcuda_gemm_hmx_ex(dev, hi, V, 0, nullptr, nullptr, HEXCUDA_HMX_RES_NONE, nullptr, ahi,
                                     HEXCUDA_HMX_STORE_ACC_I32, HEXCUDA_HMX_ACT_NONE, 0, SQ, D, SK, 8))
        return rc;
    launch_begin(d);
    combine_field_kernel<<<grid_for(d, sd), 256, 0, d->stream>>>(ahi, alo, out, sd);
    return launch_end(d, "attn_qkt_av_hmx combine");
}
