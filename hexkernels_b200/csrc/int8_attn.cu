// int8_attn.cu -- the corpus's int8 attention blocks with the LUT softmax:
//
//   gqa_attention            Q, K, V int8; scores = requant_i8(QK^T); probs
//                            from the exp table; out int8 = requant_i8(PV)
//                            (kernels/expert/gqa_attention/reference.c)
//   i8_attention_block,      Q u8, K / V int8; scores = clamp_i8(sx12(HMX
//   i8_gqa_attention_block   field of QK^T) >> 4); out uint16 = HMX field of PV
//                            (i8_attention_block/reference.c,
//                            i8_gqa_attention_block/reference.c)
//   i8_rope_attention_block  the same after rotating Q and K with int8 cos /
//                            sin tables (i8_rope_attention_block/reference.c)
//   i8_decoder_block         causal self-attention of X (u8) with itself,
//                            residual, then a two-layer int8 FFN with a LUT
//                            activation (i8_decoder_block/reference.c)
//
// LUT softmax of a score row (identical in all five): m = row max; e_j =
// exp_lut[max(s_j - m, -255) + 255]; S = sum e_j; p_j = (e_j * 255 + S / 2) / S.
//
// These blocks are small (sequence and head sizes of tens): one CTA per query
// head keeps the head's Q, K, V, scores and probabilities in shared memory
// and computes every dot product with dp4a (four byte products per
// instruction); a tensor-core pipeline would spend more in set-up than the
// work takes.  All arithmetic is integer, so results are bit-exact.
#include "hx_internal.h"

namespace hx {
namespace {

enum { kModeRq = 0, kModeHmx = 1, kModeRope = 2 };
constexpr int kThreads = 256;

struct AttnI8Args {
    const void *Q;
    const int8_t *K, *V;
    const uint8_t *exp_lut;
    const int8_t *cos_lut, *sin_lut;
    int rot_shift;
    void *out;
    int HQ, HKV, S, D;
    int32_t smult, amult;
    int sshift, ashift;
    int window;   // REQUANT mode: scores with |i - j| > window become -128 (< 0: none)
};

// 4-byte dot products: d = c + sum a_i * b_i over the bytes of a and b
__device__ __forceinline__ int dot_us(uint32_t a, uint32_t b, int c) {   // a u8, b s8
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dot_ss(uint32_t a, uint32_t b, int c) {   // both s8
    return __dp4a((int)a, (int)b, c);
}
__device__ __forceinline__ int dot_uu(uint32_t a, uint32_t b, int c) {   // both u8
    return (int)__dp4a(a, b, (unsigned)c);
}

__device__ __forceinline__ int clamp_i8(int v) { return v > 127 ? 127 : (v < -128 ? -128 : v); }
__device__ __forceinline__ int clamp_u8(int v) { return v > 255 ? 255 : (v < 0 ? 0 : v); }

// requant_i8 of gqa_attention/reference.c: round half away from zero, no zp
__device__ __forceinline__ int requant_i8(int32_t raw, int32_t mult, int shift) {
    const int64_t v = (int64_t)raw * (int64_t)mult;
    const int64_t half = shift > 0 ? ((int64_t)1 << (shift - 1)) : 0;
    int64_t q = v >= 0 ? ((v + half) >> shift) : -(((-v) + half) >> shift);
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    return (int)q;
}

// the HMX 0x40 requant field: ((acc * 17 + 8) >> 4) & 0xFFF (int wrap)
__device__ __forceinline__ int hmx_field(int acc) {
    return ((int)((uint32_t)acc * 17u + 8u) >> 4) & 0xFFF;
}
__device__ __forceinline__ int sx12(int f) { return (int)((uint32_t)f << 20) >> 20; }

// Row softmax through the exp table over the first `n` of a row's columns
// (the rest of the padded row is set to 0); one warp per row.
__device__ void lut_softmax_rows(const int8_t *sc, uint8_t *pr, int S, int Sp, int causal,
                                 const uint8_t *exp_lut) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = warp; i < S; i += nw) {
        const int n = causal ? i + 1 : S;
        const int8_t *row = sc + (size_t)i * Sp;
        uint8_t *p = pr + (size_t)i * Sp;
        int m = -128;
        for (int j = lane; j < n; j += 32) m = max(m, (int)row[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        int sum = 0;
        for (int j = lane; j < n; j += 32) {
            const int diff = max((int)row[j] - m, -255);
            sum += __ldg(exp_lut + diff + 255);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const int half = sum / 2;
        for (int j = lane; j < Sp; j += 32) {
            int v = 0;
            if (j < n && sum > 0) {
                const int e = __ldg(exp_lut + max((int)row[j] - m, -255) + 255);
                v = (e * 255 + half) / sum;
            }
            p[j] = (uint8_t)v;
        }
    }
}

__host__ __device__ inline int round4(int x) { return (x + 3) & ~3; }

// shared-memory plan of the attention kernel (bytes)
struct AttnSmem {
    int Sp, Dp, q, k, vt, sc, pr, total;
    __host__ __device__ AttnSmem(int S, int D) {
        Sp = round4(S);
        Dp = round4(D);
        q = 0;
        k = q + S * Dp;
        vt = k + S * Dp;
        sc = vt + Dp * Sp;
        pr = sc + S * Sp;
        total = (pr + S * Sp + 15) & ~15;
    }
};

template <int MODE>
__global__ void __launch_bounds__(kThreads) attn_lut_i8_kernel(const AttnI8Args a) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int hq = blockIdx.x;
    const int hkv = hq / (a.HQ / a.HKV);
    const int S = a.S, D = a.D;
    const AttnSmem L(S, D);
    const int Sp = L.Sp, Dp = L.Dp, half_d = D / 2;
    uint8_t *Qs = sm + L.q;
    int8_t *Ks = reinterpret_cast<int8_t *>(sm + L.k);
    int8_t *Vt = reinterpret_cast<int8_t *>(sm + L.vt);
    int8_t *sc = reinterpret_cast<int8_t *>(sm + L.sc);
    uint8_t *pr = sm + L.pr;
    const uint8_t *Qg = reinterpret_cast<const uint8_t *>(a.Q) + (size_t)hq * S * D;
    const int8_t *Kg = a.K + (size_t)hkv * S * D;
    const int8_t *Vg = a.V + (size_t)hkv * S * D;
    // operands into shared memory, rows padded with zeros to 4 bytes (zeros
    // add nothing to the dot products); V transposed so PV reads rows too
    for (int idx = threadIdx.x; idx < S * Dp; idx += blockDim.x) {
        const int i = idx / Dp, d = idx % Dp;
        uint8_t q = 0;
        int8_t k = 0;
        if (d < D) {
            if constexpr (MODE == kModeRope) {
                // rotate pairs (d, d + D/2) by the row's int8 cos / sin
                const int dd = d < half_d ? d : d - half_d;
                if (dd < half_d) {
                    const int c = a.cos_lut[i * half_d + dd], s = a.sin_lut[i * half_d + dd];
                    const int q0 = Qg[i * D + dd], q1 = Qg[i * D + dd + half_d];
                    const int k0 = Kg[i * D + dd], k1 = Kg[i * D + dd + half_d];
                    if (d < half_d) {
                        q = (uint8_t)clamp_u8((q0 * c - q1 * s) >> a.rot_shift);
                        k = (int8_t)clamp_i8((k0 * c - k1 * s) >> a.rot_shift);
                    } else {
                        q = (uint8_t)clamp_u8((q0 * s + q1 * c) >> a.rot_shift);
                        k = (int8_t)clamp_i8((k0 * s + k1 * c) >> a.rot_shift);
                    }
                }
            } else {
                q = Qg[i * D + d];
                k = Kg[i * D + d];
            }
        }
        Qs[i * Dp + d] = q;
        Ks[i * Dp + d] = k;
    }
    for (int idx = threadIdx.x; idx < Dp * Sp; idx += blockDim.x) {
        const int d = idx / Sp, j = idx % Sp;
        Vt[idx] = (d < D && j < S) ? Vg[j * D + d] : (int8_t)0;
    }
    __syncthreads();
    // scores
    for (int idx = threadIdx.x; idx < S * Sp; idx += blockDim.x) {
        const int i = idx / Sp, j = idx % Sp;
        int v = 0;
        if (j < S) {
            const uint32_t *qr = reinterpret_cast<const uint32_t *>(Qs + i * Dp);
            const uint32_t *kr = reinterpret_cast<const uint32_t *>(Ks + j * Dp);
            int acc = 0;
            for (int w = 0; w < Dp / 4; w++)
                acc = MODE == kModeRq ? dot_ss(qr[w], kr[w], acc) : dot_us(qr[w], kr[w], acc);
            v = MODE == kModeRq ? requant_i8(acc, a.smult, a.sshift)
                                : clamp_i8(sx12(hmx_field(acc)) >> 4);
            // banded mask of i8_sparse_attn_block/reference.c:33-42: the
            // masked scores stay in the softmax at the int8 minimum
            if (MODE == kModeRq && a.window >= 0 && abs(i - j) > a.window) v = -128;
        }
        sc[idx] = (int8_t)v;
    }
    __syncthreads();
    lut_softmax_rows(sc, pr, S, Sp, 0, a.exp_lut);
    __syncthreads();
    // P V
    for (int idx = threadIdx.x; idx < S * D; idx += blockDim.x) {
        const int i = idx / D, d = idx % D;
        const uint32_t *pp = reinterpret_cast<const uint32_t *>(pr + i * Sp);
        const uint32_t *vv = reinterpret_cast<const uint32_t *>(Vt + d * Sp);
        int acc = 0;
        for (int w = 0; w < Sp / 4; w++) acc = dot_us(pp[w], vv[w], acc);
        const size_t o = (size_t)hq * S * D + idx;
        if constexpr (MODE == kModeRq)
            reinterpret_cast<int8_t *>(a.out)[o] = (int8_t)requant_i8(acc, a.amult, a.ashift);
        else
            reinterpret_cast<uint16_t *>(a.out)[o] = (uint16_t)hmx_field(acc);
    }
}

// shared-memory plan of the decoder block kernel (bytes)
struct DecSmem {
    int Sp, Dp, Fp, xs, xt, sc, pr, hs, w1t, ha, w2t, total;
    __host__ __device__ DecSmem(int S, int D, int Dff) {
        Sp = round4(S);
        Dp = round4(D);
        Fp = round4(Dff);
        xs = 0;
        xt = xs + S * Dp;
        sc = xt + Dp * Sp;
        pr = sc + S * Sp;
        hs = pr + S * Sp;
        w1t = hs + S * Dp;
        ha = w1t + Dff * Dp;
        w2t = ha + S * Fp;
        total = (w2t + D * Fp + 15) & ~15;
    }
};

struct DecArgs {
    const uint8_t *X;
    const int8_t *W1, *W2, *act_lut;
    const int32_t *b1, *b2;
    const uint8_t *exp_lut;
    int8_t *out;
    int S, D, Dff;
};

// i8_decoder_block/kernel_api.h:48-51
constexpr int kAttnScaleShift = 2, kAttnOutShift = 8, kFfnSh1 = 8, kFfnSh2 = 7;
// i8_transformer_encoder_block/kernel_api.h:45-48
constexpr int kEncScaleShift = 4, kEncOutShift = 8, kEncSh1 = 8, kEncSh2 = 4;

// ENC false: i8_decoder_block (causal, plain shifts, table activation).
// ENC true: i8_transformer_encoder_block (reference.c:18-78): every key,
// X read as u8 on the query side and as int8 on the key / value side, HMX
// 12-bit fields after each product, ReLU + shift between the FFN layers,
// and the second residual added after the shift without saturating first.
template <bool ENC>
__global__ void __launch_bounds__(kThreads) block_i8_kernel(const DecArgs a) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int S = a.S, D = a.D, F = a.Dff;
    const DecSmem L(S, D, F);
    const int Sp = L.Sp, Dp = L.Dp, Fp = L.Fp;
    uint8_t *Xs = sm + L.xs, *Xt = sm + L.xt, *pr = sm + L.pr, *hs = sm + L.hs;
    int8_t *sc = reinterpret_cast<int8_t *>(sm + L.sc);
    int8_t *W1t = reinterpret_cast<int8_t *>(sm + L.w1t);
    int8_t *Ha = reinterpret_cast<int8_t *>(sm + L.ha);
    int8_t *W2t = reinterpret_cast<int8_t *>(sm + L.w2t);
    for (int idx = threadIdx.x; idx < S * Dp; idx += blockDim.x) {
        const int i = idx / Dp, d = idx % Dp;
        Xs[idx] = d < D ? a.X[i * D + d] : (uint8_t)0;
    }
    for (int idx = threadIdx.x; idx < Dp * Sp; idx += blockDim.x) {
        const int d = idx / Sp, j = idx % Sp;
        Xt[idx] = (d < D && j < S) ? a.X[j * D + d] : (uint8_t)0;
    }
    for (int idx = threadIdx.x; idx < F * Dp; idx += blockDim.x) {   // W1 [D][F] -> [F][Dp]
        const int j = idx / Dp, k = idx % Dp;
        W1t[idx] = k < D ? a.W1[k * F + j] : (int8_t)0;
    }
    for (int idx = threadIdx.x; idx < D * Fp; idx += blockDim.x) {   // W2 [F][D] -> [D][Fp]
        const int j = idx / Fp, k = idx % Fp;
        W2t[idx] = k < F ? a.W2[k * D + j] : (int8_t)0;
    }
    __syncthreads();
    // scores: causal (key j <= query i) for the decoder, every key for the encoder
    for (int idx = threadIdx.x; idx < S * Sp; idx += blockDim.x) {
        const int i = idx / Sp, j = idx % Sp;
        int v = 0;
        if (ENC ? j < S : j <= i) {
            const uint32_t *xi = reinterpret_cast<const uint32_t *>(Xs + i * Dp);
            const uint32_t *xj = reinterpret_cast<const uint32_t *>(Xs + j * Dp);
            int raw = 0;
            if constexpr (ENC) {
                for (int w = 0; w < Dp / 4; w++) raw = dot_us(xi[w], xj[w], raw);
                v = clamp_i8(sx12(hmx_field(raw)) >> kEncScaleShift);
            } else {
                for (int w = 0; w < Dp / 4; w++) raw = dot_uu(xi[w], xj[w], raw);
                v = clamp_i8(raw >> kAttnScaleShift);
            }
        }
        sc[idx] = (int8_t)v;
    }
    __syncthreads();
    lut_softmax_rows(sc, pr, S, Sp, ENC ? 0 : 1, a.exp_lut);
    __syncthreads();
    // attention output and residual: h = clamp_u8(X + clamp_i8(P X >> 8))
    for (int idx = threadIdx.x; idx < S * Dp; idx += blockDim.x) {
        const int i = idx / Dp, d = idx % Dp;
        uint8_t h = 0;
        if (d < D) {
            const uint32_t *pp = reinterpret_cast<const uint32_t *>(pr + i * Sp);
            const uint32_t *xx = reinterpret_cast<const uint32_t *>(Xt + d * Sp);
            int av = 0;
            int at;
            if constexpr (ENC) {
                for (int w = 0; w < Sp / 4; w++) av = dot_us(pp[w], xx[w], av);
                at = clamp_i8(sx12(hmx_field(av)) >> kEncOutShift);
            } else {
                for (int w = 0; w < Sp / 4; w++) av = dot_uu(pp[w], xx[w], av);
                at = clamp_i8(av >> kAttnOutShift);
            }
            h = (uint8_t)clamp_u8((int)Xs[i * Dp + d] + at);
        }
        hs[idx] = h;
    }
    __syncthreads();
    // FFN up-projection and LUT activation
    for (int idx = threadIdx.x; idx < S * Fp; idx += blockDim.x) {
        const int i = idx / Fp, j = idx % Fp;
        int8_t v = 0;
        if (j < F) {
            const uint32_t *hh = reinterpret_cast<const uint32_t *>(hs + i * Dp);
            const uint32_t *ww = reinterpret_cast<const uint32_t *>(W1t + j * Dp);
            int acc = 0;
            for (int w = 0; w < Dp / 4; w++) acc = dot_us(hh[w], ww[w], acc);
            if constexpr (ENC) {
                const int p1 = sx12(hmx_field(acc)) + a.b1[j];
                v = (int8_t)(p1 > 0 ? min(p1 >> kEncSh1, 127) : 0);
            } else {
                const int p1 = (acc >> kFfnSh1) + a.b1[j];
                v = __ldg(a.act_lut + clamp_i8(p1) + 128);
            }
        }
        Ha[idx] = v;
    }
    __syncthreads();
    // FFN down-projection, bias, saturate, residual
    for (int idx = threadIdx.x; idx < S * D; idx += blockDim.x) {
        const int i = idx / D, j = idx % D;
        const uint32_t *hh = reinterpret_cast<const uint32_t *>(Ha + i * Fp);
        const uint32_t *ww = reinterpret_cast<const uint32_t *>(W2t + j * Fp);
        int acc = 0;
        for (int w = 0; w < Fp / 4; w++) acc = dot_ss(hh[w], ww[w], acc);
        // (the encoder's hidden values are in [0, 127]: signed and unsigned
        // bytes agree)
        const int fv = ENC ? (sx12(hmx_field(acc)) + a.b2[j]) >> kEncSh2
                           : clamp_i8((acc >> kFfnSh2) + a.b2[j]);
        a.out[idx] = (int8_t)clamp_i8((int)hs[i * Dp + j] + fv);
    }
}

constexpr int kMaxSmem = 200 * 1024;

// Raise the kernel's dynamic shared-memory limit to kMaxSmem once per device
// (setting it to one launch's size would refuse later, larger launches).
template <typename K>
int set_smem(K kern, int dev_ordinal, bool *done) {
    if (done[dev_ordinal & 63]) return HEXCUDA_OK;
    if (int rc = check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem),
                       "cudaFuncSetAttribute(int8 attention)"))
        return rc;
    done[dev_ordinal & 63] = true;
    return HEXCUDA_OK;
}

}  // namespace
}  // namespace hx

using namespace hx;

namespace hx {
namespace {
int attn_lut_i8_run(int dev, int mode, const void *Q, const int8_t *K, const int8_t *V,
                    const uint8_t *exp_lut, const int8_t *cos_lut, const int8_t *sin_lut,
                    int rot_shift, void *out, int HQ, int HKV, int S, int D, int32_t scale_mult,
                    int scale_shift, int32_t av_mult, int av_shift, int window) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (mode < HEXCUDA_ATTN_LUT_REQUANT || mode > HEXCUDA_ATTN_LUT_HMX_ROPE || HQ < 1 || HKV < 1 ||
        HQ % HKV != 0 || S < 0 || D < 0)
        return fail(HEXCUDA_ERR_ARG, "attn_lut_i8: mode %d heads %d/%d S %d D %d", mode, HQ, HKV, S, D);
    if (mode == HEXCUDA_ATTN_LUT_REQUANT &&
        (scale_shift < 0 || scale_shift > 63 || av_shift < 0 || av_shift > 63))
        return fail(HEXCUDA_ERR_ARG, "attn_lut_i8: shifts %d / %d (0..63)", scale_shift, av_shift);
    if (mode == HEXCUDA_ATTN_LUT_HMX_ROPE && (D % 2 || rot_shift < 0 || rot_shift > 31))
        return fail(HEXCUDA_ERR_ARG, "attn_lut_i8: rotation needs even D and shift 0..31");
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (!Q || !K || !V || !exp_lut || !out ||
        (mode == HEXCUDA_ATTN_LUT_HMX_ROPE && (!cos_lut || !sin_lut)))
        return fail(HEXCUDA_ERR_ARG, "attn_lut_i8: null pointer");
    const AttnSmem L(S, D);
    if (L.total > kMaxSmem)
        return fail(HEXCUDA_ERR_ARG, "attn_lut_i8: S=%d D=%d need %d B of shared memory (max %d)", S,
                    D, L.total, kMaxSmem);
    AttnI8Args a{Q, K, V, exp_lut, cos_lut, sin_lut, rot_shift, out, HQ, HKV, S, D,
                 scale_mult, av_mult, scale_shift, av_shift, window};
    static bool done[3][64] = {};
    launch_begin(d);
    int rc;
    if (mode == HEXCUDA_ATTN_LUT_REQUANT) {
        if (!(rc = set_smem(attn_lut_i8_kernel<kModeRq>, d->ordinal, done[0])))
            attn_lut_i8_kernel<kModeRq><<<HQ, kThreads, L.total, d->stream>>>(a);
    } else if (mode == HEXCUDA_ATTN_LUT_HMX) {
        if (!(rc = set_smem(attn_lut_i8_kernel<kModeHmx>, d->ordinal, done[1])))
            attn_lut_i8_kernel<kModeHmx><<<HQ, kThreads, L.total, d->stream>>>(a);
    } else {
        if (!(rc = set_smem(attn_lut_i8_kernel<kModeRope>, d->ordinal, done[2])))
            attn_lut_i8_kernel<kModeRope><<<HQ, kThreads, L.total, d->stream>>>(a);
    }
    if (rc) return rc;
    return launch_end(d, "attn_lut_i8");
}
}  // namespace
}  // namespace hx

HX_EXPORT int hexcuda_attn_lut_i8(int dev, int mode, const void *Q, const int8_t *K, const int8_t *V,
                                  const uint8_t *exp_lut, const int8_t *cos_lut,
                                  const int8_t *sin_lut, int rot_shift, void *out, int HQ, int HKV,
                                  int S, int D, int32_t scale_mult, int scale_shift, int32_t av_mult,
                                  int av_shift) {
    return attn_lut_i8_run(dev, mode, Q, K, V, exp_lut, cos_lut, sin_lut, rot_shift, out, HQ, HKV, S,
                           D, scale_mult, scale_shift, av_mult, av_shift, -1);
}

HX_EXPORT int hexcuda_attn_lut_i8_window(int dev, const int8_t *Q, const int8_t *K, const int8_t *V,
                                         const uint8_t *exp_lut, int8_t *out, int H, int S, int D,
                                         int window, int32_t scale_mult, int scale_shift,
                                         int32_t av_mult, int av_shift) {
    if (window < 0) return fail(HEXCUDA_ERR_ARG, "attn_lut_i8_window: window %d", window);
    return attn_lut_i8_run(dev, HEXCUDA_ATTN_LUT_REQUANT, Q, K, V, exp_lut, nullptr, nullptr, 0, out,
                           H, H, S, D, scale_mult, scale_shift, av_mult, av_shift, window);
}

HX_EXPORT int hexcuda_decoder_block_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                       const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                                       const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (S < 0 || D < 0 || Dff < 0)
        return fail(HEXCUDA_ERR_ARG, "decoder_block_i8: S %d D %d Dff %d", S, D, Dff);
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (!X || !W1 || !b1 || !act_lut || !W2 || !b2 || !exp_lut || !out)
        return fail(HEXCUDA_ERR_ARG, "decoder_block_i8: null pointer");
    const DecSmem L(S, D, Dff);
    if (L.total > kMaxSmem)
        return fail(HEXCUDA_ERR_ARG, "decoder_block_i8: S=%d D=%d Dff=%d need %d B of shared memory",
                    S, D, Dff, L.total);
    DecArgs a{X, W1, W2, act_lut, b1, b2, exp_lut, out, S, D, Dff};
    static bool done[64] = {};
    launch_begin(d);
    if (int rc = set_smem(block_i8_kernel<false>, d->ordinal, done)) return rc;
    block_i8_kernel<false><<<1, kThreads, L.total, d->stream>>>(a);
    return launch_end(d, "decoder_block_i8");
}

HX_EXPORT int hexcuda_encoder_block_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                       const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut,
                                       int8_t *out, int S, int D, int Dff) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (S < 0 || D < 0 || Dff < 0)
        return fail(HEXCUDA_ERR_ARG, "encoder_block_i8: S %d D %d Dff %d", S, D, Dff);
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (!X || !W1 || !b1 || !W2 || !b2 || !exp_lut || !out)
        return fail(HEXCUDA_ERR_ARG, "encoder_block_i8: null pointer");
    const DecSmem L(S, D, Dff);
    if (L.total > kMaxSmem)
        return fail(HEXCUDA_ERR_ARG, "encoder_block_i8: S=%d D=%d Dff=%d need %d B of shared memory",
                    S, D, Dff, L.total);
    DecArgs a{X, W1, W2, nullptr, b1, b2, exp_lut, out, S, D, Dff};
    static bool done[64] = {};
    launch_begin(d);
    if (int rc = set_smem(block_i8_kernel<true>, d->ordinal, done)) return rc;
    block_i8_kernel<true><<<1, kThreads, L.total, d->stream>>>(a);
    return launch_end(d, "encoder_block_i8");
}
