/* hexoracle.c -- CPU oracle for the hot-path operators (TEST INFRASTRUCTURE).
 *
 * The checker for the CUDA path, never the product.  Each function restates
 * one scalar reference.c of sriharshapy/hexkernels (cited per function) with
 * the same arithmetic, accumulation order and rounding.  Parity of this file
 * with the reference itself is pinned by the golden vectors in tests/golden/,
 * produced by the reference's own reference.c files (see oracle/Makefile).
 */
#include "hexoracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline float h2f(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}
static inline uint16_t f2h(float f) {
    _Float16 h = (_Float16)f;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

/* Round-half-away-from-zero fixed-point requant shared by every integer
 * reference: i8_gemm_requant/reference.c:11-13,
 * requant_per_channel/reference.c:7-10, requantize_i32_u8_dma/reference.c:6-8. */
static inline int64_t rq_round(int64_t v, int shift) {
    int64_t half = shift > 0 ? ((int64_t)1 << (shift - 1)) : 0;
    return (v >= 0) ? ((v + half) >> shift) : -(((-v) + half) >> shift);
}
static inline int8_t sat_i8(int64_t r) {
    if (r > 127) r = 127;
    if (r < -128) r = -128;
    return (int8_t)r;
}
static inline uint8_t sat_u8(int64_t r) {
    if (r > 255) r = 255;
    if (r < 0) r = 0;
    return (uint8_t)r;
}

/* The integer GEMMs accumulate with the k loop outermost over a row of int32
 * partial sums.  Integer addition is associative, so this is bit-identical to
 * the reference's j-outer / k-inner order while letting gcc vectorise. */

/* kernels/expert/i8_gemm_requant/reference.c:5-19 */
void oracle_i8_gemm_requant_rows(const int8_t *A, const int8_t *B, int8_t *out,
                                 int M, int N, int K, int32_t mult, int shift,
                                 int8_t zp, int r0, int r1) {
    (void)M;
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)N);
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(int32_t) * (size_t)N);
        for (int k = 0; k < K; k++) {
            int32_t a = A[(size_t)i * K + k];
            const int8_t *b = B + (size_t)k * N;
            for (int j = 0; j < N; j++) acc[j] += a * (int32_t)b[j];
        }
        for (int j = 0; j < N; j++) {
            int64_t v = (int64_t)acc[j] * (int64_t)mult;
            int64_t r = rq_round(v, shift) + zp;
            out[(size_t)i * N + j] = sat_i8(r);
        }
    }
    free(acc);
}

/* kernels/expert/i8_gemm_bias_requant/reference.c:6-22 */
void oracle_i8_gemm_bias_requant_rows(const int8_t *A, const int8_t *B,
                                      const int32_t *bias, int8_t *out,
                                      int M, int N, int K, int32_t mult,
                                      int shift, int8_t zp, int r0, int r1) {
    (void)M;
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)N);
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(int32_t) * (size_t)N);
        for (int k = 0; k < K; k++) {
            int32_t a = A[(size_t)i * K + k];
            const int8_t *b = B + (size_t)k * N;
            for (int j = 0; j < N; j++) acc[j] += a * (int32_t)b[j];
        }
        for (int j = 0; j < N; j++) {
            int64_t biased = (int64_t)acc[j] + (int64_t)bias[j];
            int64_t v = biased * (int64_t)mult;
            out[(size_t)i * N + j] = sat_i8(rq_round(v, shift) + zp);
        }
    }
    free(acc);
}

/* kernels/expert/gemm_tile_zp_i8/reference.c:10-29.  colsum and the
 * zpA * colsum product are int32 exactly as the reference computes them
 * (two's-complement wrap where the C would overflow). */
void oracle_gemm_tile_zp_i8_rows(const int8_t *A, const int8_t *B, int8_t *out,
                                 int M, int N, int K, int32_t zpA,
                                 int32_t scale_mult, int scale_shift,
                                 int r0, int r1) {
    (void)M;
    int32_t *colsum = (int32_t *)calloc((size_t)N, sizeof(int32_t));
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)N);
    for (int k = 0; k < K; k++)
        for (int j = 0; j < N; j++) colsum[j] += (int32_t)B[(size_t)k * N + j];
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(int32_t) * (size_t)N);
        for (int k = 0; k < K; k++) {
            int32_t a = A[(size_t)i * K + k];
            const int8_t *b = B + (size_t)k * N;
            for (int j = 0; j < N; j++) acc[j] += a * (int32_t)b[j];
        }
        for (int j = 0; j < N; j++) {
            int32_t zc = (int32_t)((uint32_t)zpA * (uint32_t)colsum[j]);
            int32_t a32 = (int32_t)((uint32_t)acc[j] - (uint32_t)zc);
            int64_t r = (int64_t)a32 * (int64_t)scale_mult;
            out[(size_t)i * N + j] = sat_i8(rq_round(r, scale_shift));
        }
    }
    free(acc);
    free(colsum);
}

/* Composed u8 x s8 per-channel GEMM (see header for the four cited lines). */
void oracle_gemm_u8s8_pc_rows(const uint8_t *A, const int8_t *B,
                              const int32_t *bias, uint8_t *out,
                              int M, int N, int K, int32_t zpA,
                              const int32_t *mult, const int *shift,
                              uint8_t zp_out, int r0, int r1) {
    (void)M;
    int32_t *colsum = (int32_t *)calloc((size_t)N, sizeof(int32_t));
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)N);
    for (int k = 0; k < K; k++)
        for (int j = 0; j < N; j++) colsum[j] += (int32_t)B[(size_t)k * N + j];
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(int32_t) * (size_t)N);
        for (int k = 0; k < K; k++) {
            int32_t a = A[(size_t)i * K + k];
            const int8_t *b = B + (size_t)k * N;
            for (int j = 0; j < N; j++) acc[j] += a * (int32_t)b[j];
        }
        for (int j = 0; j < N; j++) {
            int32_t zc = (int32_t)((uint32_t)zpA * (uint32_t)colsum[j]);
            int32_t a32 = (int32_t)((uint32_t)acc[j] - (uint32_t)zc);
            int64_t biased = (int64_t)a32 + (int64_t)bias[j];
            int64_t v = biased * (int64_t)mult[j];
            int64_t r = rq_round(v, shift[j]) + (int64_t)zp_out;
            out[(size_t)i * N + j] = sat_u8(r);
        }
    }
    free(acc);
    free(colsum);
}

/* sx12 of the HMX references (e.g. hmx_matmul_i8_64/reference.c:4):
 * low 12 bits, sign-extended. */
static inline int32_t sx12(int32_t f) {
    int32_t v = f & 0xFFF;
    if (v & 0x800) v -= 0x1000;
    return v;
}

static inline int32_t wrap_add(int32_t a, int32_t b) {
    return (int32_t)((uint32_t)a + (uint32_t)b);
}

/* The HMX-convention references (cited in hexoracle.h).  acc is the int32
 * sum of (A - zpA) * B in k order with two's-complement wrap; the
 * (acc * 17 + 8) >> 4 step and the later int adds are the references' int
 * arithmetic as gcc compiles it (wrap, arithmetic shift). */
void oracle_gemm_hmx_ex_rows(const uint8_t *A, const int8_t *B, int b_transposed,
                             void *out, int M, int N, int K, int32_t zpA, int store,
                             int act, const int32_t *bias, int res_kind, const void *res,
                             const void *lut, int col_major, int r0, int r1) {
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)(N > 0 ? N : 1));
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(int32_t) * (size_t)N);
        for (int k = 0; k < K; k++) {
            const uint32_t a = (uint32_t)((int32_t)A[(size_t)i * K + k] - zpA);
            if (b_transposed) {
                for (int j = 0; j < N; j++)
                    acc[j] = (int32_t)((uint32_t)acc[j] + a * (uint32_t)(int32_t)B[(size_t)j * K + k]);
            } else {
                const int8_t *b = B + (size_t)k * N;
                for (int j = 0; j < N; j++)
                    acc[j] = (int32_t)((uint32_t)acc[j] + a * (uint32_t)(int32_t)b[j]);
            }
        }
        for (int j = 0; j < N; j++) {
            const int32_t f = (int32_t)((uint32_t)acc[j] * 17u + 8u) >> 4;
            int32_t v = store == ORACLE_HMX_STORE_ACC_I32 ? acc[j] : sx12(f);
            const size_t rm = (size_t)i * N + j;
            if (bias) v = wrap_add(v, bias[j]);
            if (res_kind == ORACLE_HMX_RES_I32) v = wrap_add(v, ((const int32_t *)res)[rm]);
            if (res_kind == ORACLE_HMX_RES_I8) v = wrap_add(v, ((const int8_t *)res)[rm]);
            if (act == ORACLE_HMX_ACT_RELU) v = v > 0 ? v : 0;
            if (act == ORACLE_HMX_ACT_LEAKY_SHR3) v = v >= 0 ? v : (v >> 3);
            const size_t o = col_major ? (size_t)j * M + i : rm;
            switch (store) {
            case ORACLE_HMX_STORE_I32:
            case ORACLE_HMX_STORE_ACC_I32: ((int32_t *)out)[o] = v; break;
            case ORACLE_HMX_STORE_I8_SAT: ((int8_t *)out)[o] = sat_i8(v); break;
            case ORACLE_HMX_STORE_U8_SAT: ((uint8_t *)out)[o] = sat_u8(v); break;
            case ORACLE_HMX_STORE_I8_LOW: ((int8_t *)out)[o] = (int8_t)(uint8_t)(v & 0xFF); break;
            case ORACLE_HMX_STORE_U16_FIELD: ((uint16_t *)out)[o] = (uint16_t)(v & 0xFFF); break;
            case ORACLE_HMX_STORE_LUT_I32: {
                /* hmx_matmul_i8_gelu_lut/reference.c: lut[r + 128]; the
                 * reference is undefined outside the table, here clamped */
                int32_t ix = v + 128;
                ix = ix < 0 ? 0 : (ix > 255 ? 255 : ix);
                ((int32_t *)out)[o] = ((const int32_t *)lut)[ix];
                break;
            }
            case ORACLE_HMX_STORE_LUT_I8:
                /* i8_matmul_bias_gelu_hmx/reference.c: lut[(uint8)(sat_i8 + 128)] */
                ((int8_t *)out)[o] = ((const int8_t *)lut)[(uint8_t)(sat_i8(v) + 128)];
                break;
            default: break;
            }
        }
    }
    free(acc);
}

void oracle_gemm_hmx_rows(const uint8_t *A, const int8_t *B, int b_transposed,
                          const int32_t *bias, void *out, int M, int N, int K,
                          int32_t zpA, int mode, int r0, int r1) {
    if (mode == 0)
        oracle_gemm_hmx_ex_rows(A, B, b_transposed, out, M, N, K, zpA, ORACLE_HMX_STORE_I32,
                                ORACLE_HMX_ACT_NONE, 0, 0, 0, 0, 0, r0, r1);
    else if (mode == 1)
        oracle_gemm_hmx_ex_rows(A, B, b_transposed, out, M, N, K, zpA, ORACLE_HMX_STORE_I8_SAT,
                                ORACLE_HMX_ACT_NONE, 0, 0, 0, 0, 0, r0, r1);
    else
        oracle_gemm_hmx_ex_rows(A, B, b_transposed, out, M, N, K, zpA, ORACLE_HMX_STORE_U8_SAT,
                                ORACLE_HMX_ACT_RELU, bias, 0, 0, 0, 0, r0, r1);
}

void oracle_attn_qkt_av_hmx(const uint8_t *Q, const int8_t *K, const int8_t *V, int32_t *out,
                            int SQ, int SK, int D) {
    int32_t *sc = (int32_t *)malloc(sizeof(int32_t) * (size_t)(SK > 0 ? SK : 1));
    for (int i = 0; i < SQ; i++) {
        for (int j = 0; j < SK; j++) {
            uint32_t acc = 0;
            for (int d = 0; d < D; d++)
                acc += (uint32_t)((int32_t)Q[(size_t)i * D + d] * (int32_t)K[(size_t)j * D + d]);
            sc[j] = sx12((int32_t)(acc * 17u + 8u) >> 4);
        }
        for (int d = 0; d < D; d++) {
            uint32_t acc = 0;
            for (int j = 0; j < SK; j++) acc += (uint32_t)(sc[j] * (int32_t)V[(size_t)j * D + d]);
            out[(size_t)i * D + d] = sx12((int32_t)(acc * 17u + 8u) >> 4);
        }
    }
    free(sc);
}

static int clamp_i8i(int v) { return v > 127 ? 127 : (v < -128 ? -128 : v); }
static int clamp_u8i(int v) { return v > 255 ? 255 : (v < 0 ? 0 : v); }

/* gqa_attention/reference.c: requant_i8 (round half away, no zero point) */
static int requant_i8_att(int32_t raw, int32_t mult, int shift) {
    int64_t v = (int64_t)raw * (int64_t)mult;
    const int64_t q = rq_round(v, shift);
    return q > 127 ? 127 : (q < -128 ? -128 : (int)q);
}

/* the LUT softmax shared by the attention blocks, over the first n entries of
 * a row (entries n.. are set to 0) */
static void lut_softmax_row(const int8_t *row, uint8_t *p, int n, int width, const uint8_t *lut) {
    int m = row[0];
    for (int j = 1; j < n; j++) if (row[j] > m) m = row[j];
    int sum = 0;
    for (int j = 0; j < n; j++) {
        int diff = row[j] - m;
        if (diff < -255) diff = -255;
        p[j] = lut[diff + 255];
        sum += p[j];
    }
    const int half = sum / 2;
    for (int j = 0; j < n; j++) p[j] = sum > 0 ? (uint8_t)(((int)p[j] * 255 + half) / sum) : 0;
    for (int j = n; j < width; j++) p[j] = 0;
}

static int hmx_field_i(int acc) { return ((int)((uint32_t)acc * 17u + 8u) >> 4) & 0xFFF; }

static void attn_lut_i8_impl(int mode, const void *Q, const int8_t *K, const int8_t *V,
                             const uint8_t *exp_lut, const int8_t *cos_lut, const int8_t *sin_lut,
                             int rot_shift, void *out, int HQ, int HKV, int S, int D,
                             int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift,
                             int window) {
    const int group = HQ / HKV, half_d = D / 2;
    int8_t *sc = (int8_t *)malloc((size_t)S * S);
    uint8_t *pr = (uint8_t *)malloc((size_t)S * S);
    uint8_t *qr = (uint8_t *)malloc((size_t)S * D);
    int8_t *kr = (int8_t *)malloc((size_t)S * D);
    for (int hq = 0; hq < HQ; hq++) {
        const int hkv = hq / group;
        const uint8_t *Qh = (const uint8_t *)Q + (size_t)hq * S * D;
        const int8_t *Qs = (const int8_t *)Q + (size_t)hq * S * D;
        const int8_t *Kh = K + (size_t)hkv * S * D, *Vh = V + (size_t)hkv * S * D;
        if (mode == 2) {
            for (int i = 0; i < S; i++)
                for (int d = 0; d < half_d; d++) {
                    const int c = cos_lut[i * half_d + d], s = sin_lut[i * half_d + d];
                    const int q0 = Qh[i * D + d], q1 = Qh[i * D + d + half_d];
                    qr[i * D + d] = (uint8_t)clamp_u8i((q0 * c - q1 * s) >> rot_shift);
                    qr[i * D + d + half_d] = (uint8_t)clamp_u8i((q0 * s + q1 * c) >> rot_shift);
                    const int k0 = Kh[i * D + d], k1 = Kh[i * D + d + half_d];
                    kr[i * D + d] = (int8_t)clamp_i8i((k0 * c - k1 * s) >> rot_shift);
                    kr[i * D + d + half_d] = (int8_t)clamp_i8i((k0 * s + k1 * c) >> rot_shift);
                }
            Qh = qr;
            Kh = kr;
        }
        for (int i = 0; i < S; i++)
            for (int j = 0; j < S; j++) {
                int acc = 0;
                for (int d = 0; d < D; d++)
                    acc += (mode == 0 ? (int)Qs[i * D + d] : (int)Qh[i * D + d]) * (int)Kh[j * D + d];
                sc[i * S + j] = (int8_t)(mode == 0 ? requant_i8_att(acc, scale_mult, scale_shift)
                                                   : clamp_i8i(sx12(hmx_field_i(acc)) >> 4));
                /* i8_sparse_attn_block/reference.c:33-42: outside the band
                 * the score is MASK_VAL (-128) and stays in the softmax */
                if (window >= 0 && abs(i - j) > window) sc[i * S + j] = -128;
            }
        for (int i = 0; i < S; i++) lut_softmax_row(sc + (size_t)i * S, pr + (size_t)i * S, S, S, exp_lut);
        for (int i = 0; i < S; i++)
            for (int d = 0; d < D; d++) {
                int acc = 0;
                for (int j = 0; j < S; j++) acc += (int)pr[i * S + j] * (int)Vh[j * D + d];
                const size_t o = (size_t)hq * S * D + (size_t)i * D + d;
                if (mode == 0)
                    ((int8_t *)out)[o] = (int8_t)requant_i8_att(acc, av_mult, av_shift);
                else
                    ((uint16_t *)out)[o] = (uint16_t)hmx_field_i(acc);
            }
    }
    free(sc); free(pr); free(qr); free(kr);
}

void oracle_attn_lut_i8(int mode, const void *Q, const int8_t *K, const int8_t *V,
                        const uint8_t *exp_lut, const int8_t *cos_lut, const int8_t *sin_lut,
                        int rot_shift, void *out, int HQ, int HKV, int S, int D,
                        int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift) {
    attn_lut_i8_impl(mode, Q, K, V, exp_lut, cos_lut, sin_lut, rot_shift, out, HQ, HKV, S, D,
                     scale_mult, scale_shift, av_mult, av_shift, -1);
}

/* i8_sparse_attn_block/reference.c:14-62 (H heads of SEQ x HEAD_DIM) */
void oracle_attn_lut_i8_window(const int8_t *Q, const int8_t *K, const int8_t *V,
                               const uint8_t *exp_lut, int8_t *out, int H, int S, int D, int window,
                               int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift) {
    attn_lut_i8_impl(0, Q, K, V, exp_lut, NULL, NULL, 0, out, H, H, S, D, scale_mult, scale_shift,
                     av_mult, av_shift, window);
}

void oracle_decoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                             const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff) {
    int8_t *sc = (int8_t *)calloc((size_t)S * S, 1);
    uint8_t *pr = (uint8_t *)calloc((size_t)S * S, 1);
    uint8_t *h = (uint8_t *)malloc((size_t)S * D);
    int8_t *ha = (int8_t *)malloc((size_t)S * (Dff > 0 ? Dff : 1));
    for (int i = 0; i < S; i++) {
        for (int j = 0; j <= i; j++) {
            int raw = 0;
            for (int d = 0; d < D; d++) raw += (int)X[i * D + d] * (int)X[j * D + d];
            sc[i * S + j] = (int8_t)clamp_i8i(raw >> 2);
        }
        lut_softmax_row(sc + (size_t)i * S, pr + (size_t)i * S, i + 1, S, exp_lut);
        for (int d = 0; d < D; d++) {
            int av = 0;
            for (int j = 0; j <= i; j++) av += (int)pr[i * S + j] * (int)X[j * D + d];
            h[i * D + d] = (uint8_t)clamp_u8i((int)X[i * D + d] + clamp_i8i(av >> 8));
        }
    }
    for (int i = 0; i < S; i++)
        for (int j = 0; j < Dff; j++) {
            int acc = 0;
            for (int k = 0; k < D; k++) acc += (int)h[i * D + k] * (int)W1[k * Dff + j];
            ha[i * Dff + j] = act_lut[clamp_i8i((acc >> 8) + b1[j]) + 128];
        }
    for (int i = 0; i < S; i++)
        for (int j = 0; j < D; j++) {
            int acc = 0;
            for (int k = 0; k < Dff; k++) acc += (int)ha[i * Dff + k] * (int)W2[k * D + j];
            const int fv = clamp_i8i((acc >> 7) + b2[j]);
            out[i * D + j] = (int8_t)clamp_i8i((int)h[i * D + j] + fv);
        }
    free(sc); free(pr); free(h); free(ha);
}

void oracle_gemm_f16_ex_rows(const uint16_t *A, const uint16_t *B, int b_transposed,
                             const uint16_t *bias, const uint16_t *res, uint16_t *out, int M,
                             int N, int K, int act, int preround, float scale, int r0, int r1) {
    (void)M;
    for (int i = r0; i < r1; i++)
        for (int j = 0; j < N; j++) {
            /* preround 2 (fp16_matmul_bias_gelu/reference.c:16-18 and its
             * siblings): the fp32 sum of products rounded to fp16 first, then
             * residual / bias in fp32; otherwise the residual seeds the sum
             * (hmx_tile_mac_fp16_32) and the bias follows it */
            float acc = (res && preround != 2) ? h2f(res[(size_t)i * N + j]) : 0.0f;
            for (int k = 0; k < K; k++)
                acc += h2f(A[(size_t)i * K + k]) *
                       h2f(b_transposed ? B[(size_t)j * K + k] : B[(size_t)k * N + j]);
            float v = acc;
            if (preround == 2) {
                v = h2f(f2h(acc));
                if (res) v += h2f(res[(size_t)i * N + j]);
            }
            if (bias) v = v + h2f(bias[j]);
            if (preround == 1) v = h2f(f2h(v));
            if (act == 1) v = v > 0.0f ? v : 0.0f;
            if (act == 2) v = v > 0.0f ? v : v * 0.125f;
            if (act == 3) {
                const float c = 0.7978845608f * (v + 0.044715f * v * v * v);
                v = 0.5f * v * (1.0f + tanhf(c));
            }
            if (act == 4) v = 1.0f / (1.0f + expf(-v));   /* fp16_matmul_sigmoid/reference.c:4 */
            if (act == 5) v = tanhf(v);                   /* fp16_matmul_tanh/reference.c:12 */
            out[(size_t)i * N + j] = f2h(v * scale);
        }
}

void oracle_gemm_i8_rq_ex_rows(const int8_t *A, const int8_t *B, int b_transposed,
                               const int32_t *bias, const int8_t *res, int8_t *out, int M, int N,
                               int K, int32_t mult, int shift, int zp, int relu, int r0, int r1) {
    (void)M;
    for (int i = r0; i < r1; i++)
        for (int j = 0; j < N; j++) {
            uint32_t acc = 0;
            for (int k = 0; k < K; k++)
                acc += (uint32_t)((int32_t)A[(size_t)i * K + k] *
                                  (int32_t)(b_transposed ? B[(size_t)j * K + k] : B[(size_t)k * N + j]));
            int64_t x = (int64_t)(int32_t)acc + (bias ? (int64_t)bias[j] : 0);
            if (relu && x < 0) x = 0;
            int64_t q = sat_i8(rq_round(x * (int64_t)mult, shift) + zp);
            /* matmul_residual_add_i8/reference.c:19-22: + residual, saturate */
            if (res) q = sat_i8(q + res[(size_t)i * N + j]);
            out[(size_t)i * N + j] = (int8_t)q;
        }
}

void oracle_gemm_i8_acc_rows(const void *A, int a_signed, const int8_t *B, int b_transposed,
                             const int32_t *bias, const void *res, int res_kind, const void *lut,
                             void *out, int store, int act, int M, int N, int K, int r0, int r1) {
    (void)M;
    for (int i = r0; i < r1; i++)
        for (int j = 0; j < N; j++) {
            uint32_t acc = 0;
            for (int k = 0; k < K; k++) {
                const int32_t a = a_signed ? ((const int8_t *)A)[(size_t)i * K + k]
                                           : ((const uint8_t *)A)[(size_t)i * K + k];
                acc += (uint32_t)(a * (int32_t)(b_transposed ? B[(size_t)j * K + k]
                                                             : B[(size_t)k * N + j]));
            }
            int64_t x = (int64_t)(int32_t)acc + (bias ? bias[j] : 0);
            if (res_kind == ORACLE_HMX_RES_I32) x += ((const int32_t *)res)[(size_t)i * N + j];
            else if (res_kind == ORACLE_HMX_RES_I8) x += ((const int8_t *)res)[(size_t)i * N + j];
            if (act == ORACLE_HMX_ACT_RELU) x = x > 0 ? x : 0;
            else if (act == ORACLE_HMX_ACT_LEAKY_SHR3) x = x >= 0 ? x : (x >> 3);
            const size_t o = (size_t)i * N + j;
            switch (store) {
            case ORACLE_HMX_STORE_I8_SAT: ((int8_t *)out)[o] = sat_i8(x); break;
            case ORACLE_HMX_STORE_U8_SAT: ((uint8_t *)out)[o] = (uint8_t)(x > 255 ? 255 : (x < 0 ? 0 : x)); break;
            case ORACLE_HMX_STORE_I8_LOW: ((int8_t *)out)[o] = (int8_t)x; break;
            case ORACLE_HMX_STORE_U16_FIELD: ((uint16_t *)out)[o] = (uint16_t)(x & 0xFFF); break;
            case ORACLE_HMX_STORE_LUT_I32: {
                const int64_t t = x + 128 > 255 ? 255 : (x + 128 < 0 ? 0 : x + 128);
                ((int32_t *)out)[o] = ((const int32_t *)lut)[t];
                break;
            }
            case ORACLE_HMX_STORE_LUT_I8:
                ((int8_t *)out)[o] = ((const int8_t *)lut)[sat_i8(x) + 128];
                break;
            default: ((int32_t *)out)[o] = (int32_t)x; break;   /* I32, ACC_I32 */
            }
        }
}

void oracle_ffn_relu_i8(const int8_t *A, const int8_t *W1, const int32_t *b1, const int8_t *W2,
                        const int32_t *b2, int8_t *out, int M, int K, int V, int D, int32_t mult,
                        int shift, int zp) {
    int8_t *hid = (int8_t *)malloc((size_t)M * (V > 0 ? V : 1));
    oracle_gemm_i8_acc_rows(A, 1, W1, 0, b1, NULL, 0, NULL, hid, ORACLE_HMX_STORE_I8_SAT,
                            ORACLE_HMX_ACT_RELU, M, V, K, 0, M);
    oracle_gemm_i8_rq_ex_rows(hid, W2, 0, b2, NULL, out, M, D, V, mult, shift, zp, 0, 0, M);
    free(hid);
}

/* mlp_block/reference.c:19-47: the first layer through the table, the second
 * as ffn_relu_block's. */
void oracle_ffn_lut_i8(const int8_t *A, const int8_t *W1, const int32_t *b1, const int8_t *act_lut,
                       const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V, int D,
                       int32_t mult, int shift, int zp) {
    int8_t *hid = (int8_t *)malloc((size_t)M * (V > 0 ? V : 1));
    oracle_gemm_i8_acc_rows(A, 1, W1, 0, b1, NULL, 0, act_lut, hid, ORACLE_HMX_STORE_LUT_I8,
                            ORACLE_HMX_ACT_NONE, M, V, K, 0, M);
    oracle_gemm_i8_rq_ex_rows(hid, W2, 0, b2, NULL, out, M, D, V, mult, shift, zp, 0, 0, M);
    free(hid);
}

void oracle_gemm_hmx_s8u8_rows(const int8_t *A, const uint8_t *B, void *out, int store, int M,
                               int N, int K, int r0, int r1) {
    (void)M;
    for (int i = r0; i < r1; i++)
        for (int j = 0; j < N; j++) {
            uint32_t acc = 0;
            for (int k = 0; k < K; k++)
                acc += (uint32_t)((int32_t)A[(size_t)i * K + k] * (int32_t)B[(size_t)k * N + j]);
            const int32_t f = (int32_t)(acc * 17u + 8u) >> 4;
            const size_t o = (size_t)i * N + j;
            if (store == ORACLE_HMX_STORE_U16_FIELD)
                ((uint16_t *)out)[o] = (uint16_t)(f & 0xFFF);
            else if (store == ORACLE_HMX_STORE_ACC_I32)
                ((int32_t *)out)[o] = (int32_t)acc;
            else
                ((int32_t *)out)[o] = sx12(f);
        }
}

/* The elementwise requant family (cited in hexoracle.h).  Products that
 * leave int64 are undefined in the references; here they wrap. */
void oracle_requant_ew(const void *a, int a_i8, const void *b, int b_kind, int64_t n, int pre,
                       int64_t pre_c, int32_t mult, int shift, int zp, int sign_of_a,
                       int lo1, int hi1, int lo2, int hi2, const int8_t *lut, void *out) {
    const int64_t half = shift > 0 ? ((int64_t)1 << (shift - 1)) : 0;
    for (int64_t i = 0; i < n; i++) {
        const int64_t ai = a_i8 ? (int64_t)((const int8_t *)a)[i] : (int64_t)((const int32_t *)a)[i];
        int64_t bi = 0;
        if (b_kind == 1) bi = ((const int32_t *)b)[i];
        if (b_kind == 2) bi = ((const int8_t *)b)[i];
        int64_t x = ai;
        if (pre == ORACLE_RQ_PRE_ADD) x = ai + bi;
        if (pre == ORACLE_RQ_PRE_ADD_RELU) x = ai + bi > 0 ? ai + bi : 0;
        if (pre == ORACLE_RQ_PRE_MUL_ADD) x = (int64_t)((uint64_t)ai * (uint64_t)bi + (uint64_t)pre_c);
        int64_t r;
        if (sign_of_a) {
            const int64_t am = (int64_t)((uint64_t)(x < 0 ? -x : x) * (uint64_t)(int64_t)mult);
            const int64_t sh = (am + half) >> shift;
            r = x < 0 ? -sh : sh;
        } else {
            const int64_t v = (int64_t)((uint64_t)x * (uint64_t)(int64_t)mult);
            r = rq_round(v, shift);
        }
        r += zp;
        if (r > hi1) r = hi1;
        if (r < lo1) r = lo1;
        if (r > hi2) r = hi2;
        if (r < lo2) r = lo2;
        if (lut)
            ((int8_t *)out)[i] = lut[(uint8_t)r];
        else
            ((uint8_t *)out)[i] = (uint8_t)r;
    }
}

void oracle_epilogue_bias_i32(const int32_t *acc, const int32_t *bias, int32_t *out, int R, int C) {
    for (int r = 0; r < R; r++)
        for (int c = 0; c < C; c++)
            out[(size_t)r * C + c] = wrap_add(acc[(size_t)r * C + c], bias[c]);
}

void oracle_relu_i8(const int8_t *x, int8_t *out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = x[i] > 0 ? x[i] : 0;
}

/* kernels/expert/requant_per_channel/reference.c:4-16 */
void oracle_requant_per_channel(const int32_t *a, int8_t *out, int R, int C,
                                const int32_t *mult, const int *shift, int8_t zp) {
    for (int r = 0; r < R; r++) {
        int32_t m = mult[r];
        int s = shift[r];
        for (int c = 0; c < C; c++) {
            int64_t v = (int64_t)a[(size_t)r * C + c] * (int64_t)m;
            out[(size_t)r * C + c] = sat_i8(rq_round(v, s) + zp);
        }
    }
}

/* kernels/expert/requantize_i32_u8_dma/reference.c:5-18 */
void oracle_requantize_i32_u8(const int32_t *a, uint8_t *out, int64_t n,
                              int32_t mult, int shift, uint8_t zp) {
    for (int64_t i = 0; i < n; i++) {
        int64_t v = (int64_t)a[i] * (int64_t)mult;
        out[i] = sat_u8(rq_round(v, shift) + (int64_t)(uint64_t)zp);
    }
}

/* kernels/expert/fp16_attention_qkt_hmx/reference.c:8-14, M x N x K.
 * Each output keeps the reference's sequential d-order fp32 sum; the j loop
 * is innermost over a row of partial sums so it vectorises without changing
 * any element's summation order. */
void oracle_gemm_f16_nt_rows(const uint16_t *A, const uint16_t *Bt, uint16_t *out,
                             int M, int N, int K, int r0, int r1) {
    (void)M;
    float *arow = (float *)malloc(sizeof(float) * (size_t)K);
    float *acc = (float *)malloc(sizeof(float) * (size_t)N);
    float *bcol = (float *)malloc(sizeof(float) * (size_t)N * 64);
    for (int i = r0; i < r1; i++) {
        for (int d = 0; d < K; d++) arow[d] = h2f(A[(size_t)i * K + d]);
        memset(acc, 0, sizeof(float) * (size_t)N);
        for (int d0 = 0; d0 < K; d0 += 64) {
            int dn = K - d0 < 64 ? K - d0 : 64;
            for (int j = 0; j < N; j++)
                for (int dd = 0; dd < dn; dd++)
                    bcol[(size_t)dd * N + j] = h2f(Bt[(size_t)j * K + d0 + dd]);
            for (int dd = 0; dd < dn; dd++) {
                float a = arow[d0 + dd];
                const float *b = bcol + (size_t)dd * N;
                for (int j = 0; j < N; j++) acc[j] += a * b[j];
            }
        }
        for (int j = 0; j < N; j++) out[(size_t)i * N + j] = f2h(acc[j]);
    }
    free(bcol);
    free(acc);
    free(arow);
}

/* kernels/expert/hmx_matmul_fp16_deepk/reference.c:20-26, M x N x K */
void oracle_gemm_f16_nn_rows(const uint16_t *A, const uint16_t *B, uint16_t *out,
                             int M, int N, int K, int r0, int r1) {
    (void)M;
    float *acc = (float *)malloc(sizeof(float) * (size_t)N);
    for (int i = r0; i < r1; i++) {
        memset(acc, 0, sizeof(float) * (size_t)N);
        for (int k = 0; k < K; k++) {
            float a = h2f(A[(size_t)i * K + k]);
            const uint16_t *b = B + (size_t)k * N;
            for (int j = 0; j < N; j++) acc[j] += a * h2f(b[j]);
        }
        for (int j = 0; j < N; j++) out[(size_t)i * N + j] = f2h(acc[j]);
    }
    free(acc);
}

/* kernels/expert/fp16_flash_attention_tile/reference.c:11-27 for one head:
 * scores in d order, running row max seeded at -1e30f, expf, sequential row
 * sum, then per d the sequential sum over j of e[j]*V[j,d], divided once. */
void oracle_attn_f16_head_rows(const uint16_t *Q, const uint16_t *K,
                               const uint16_t *V, uint16_t *O, int SK, int D,
                               float scale, int causal, int q0, int q1) {
    float *sc = (float *)malloc(sizeof(float) * (size_t)(SK > 0 ? SK : 1));
    float *qrow = (float *)malloc(sizeof(float) * (size_t)D);
    float *acc = (float *)malloc(sizeof(float) * (size_t)D);
    for (int i = q0; i < q1; i++) {
        int nk = (causal && i + 1 < SK) ? i + 1 : SK;
        for (int d = 0; d < D; d++) qrow[d] = h2f(Q[(size_t)i * D + d]);
        float rowmax = -1e30f;
        for (int j = 0; j < nk; j++) {
            float a = 0.0f;
            const uint16_t *kr = K + (size_t)j * D;
            for (int d = 0; d < D; d++) a += qrow[d] * h2f(kr[d]);
            sc[j] = a * scale;
            if (sc[j] > rowmax) rowmax = sc[j];
        }
        float rowsum = 0.0f;
        for (int j = 0; j < nk; j++) {
            sc[j] = expf(sc[j] - rowmax);
            rowsum += sc[j];
        }
        /* acc[d] = sum_j e[j] * V[j,d] in j order for every d (same order as
         * the reference's d-outer / j-inner loop, vectorised over d). */
        for (int d = 0; d < D; d++) acc[d] = 0.0f;
        for (int j = 0; j < nk; j++) {
            float e = sc[j];
            const uint16_t *vr = V + (size_t)j * D;
            for (int d = 0; d < D; d++) acc[d] += e * h2f(vr[d]);
        }
        for (int d = 0; d < D; d++) O[(size_t)i * D + d] = f2h(acc[d] / rowsum);
    }
    free(acc);
    free(qrow);
    free(sc);
}

void oracle_attn_f16_heads(const uint16_t *Q, const uint16_t *K,
                           const uint16_t *V, uint16_t *O, int BH, int SQ,
                           int SK, int D, float scale, int causal, int h0,
                           int h1) {
    (void)BH;
    size_t qs = (size_t)SQ * D, ks = (size_t)SK * D;
    for (int h = h0; h < h1; h++)
        oracle_attn_f16_head_rows(Q + h * qs, K + h * ks, V + h * ks, O + h * qs,
                                  SK, D, scale, causal, 0, SQ);
}

/* kernels/expert/online_softmax_step_fp16/reference.c:9-37 */
void oracle_online_softmax_step_f16(const uint16_t *scores, const uint16_t *V,
                                    uint16_t *running_max, uint16_t *running_sum,
                                    uint16_t *acc, int BLK, int D) {
    float m_old = h2f(*running_max);
    float l_old = h2f(*running_sum);
    float m_blk = h2f(scores[0]);
    for (int j = 1; j < BLK; j++) {
        float v = h2f(scores[j]);
        if (v > m_blk) m_blk = v;
    }
    float m_new = (m_old > m_blk) ? m_old : m_blk;
    float corr = expf(m_old - m_new);
    float *p = (float *)malloc(sizeof(float) * (size_t)(BLK > 0 ? BLK : 1));
    float psum = 0.0f;
    for (int j = 0; j < BLK; j++) {
        p[j] = expf(h2f(scores[j]) - m_new);
        psum += p[j];
    }
    float l_new = l_old * corr + psum;
    for (int d = 0; d < D; d++) {
        float a = h2f(acc[d]) * corr;
        for (int j = 0; j < BLK; j++) a += p[j] * h2f(V[(size_t)j * D + d]);
        acc[d] = f2h(a);
    }
    *running_max = f2h(m_new);
    *running_sum = f2h(l_new);
    free(p);
}

/* kernels/expert/fp16_softmax/reference.c:9-28, fp32 storage */
void oracle_softmax_f32_rows(const float *x, float *out, int R, int C,
                             int r0, int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const float *xr = x + (size_t)r * C;
        float *outr = out + (size_t)r * C;
        float rowmax = xr[0];
        for (int j = 1; j < C; j++)
            if (xr[j] > rowmax) rowmax = xr[j];
        float rowsum = 0.0f;
        for (int j = 0; j < C; j++) {
            outr[j] = expf(xr[j] - rowmax);
            rowsum += outr[j];
        }
        for (int j = 0; j < C; j++) outr[j] = outr[j] / rowsum;
    }
}

/* kernels/expert/fp16_softmax/reference.c:9-28, fp16 storage */
void oracle_softmax_f16_rows(const uint16_t *x, uint16_t *out, int R, int C,
                             int r0, int r1) {
    (void)R;
    float *e = (float *)malloc(sizeof(float) * (size_t)(C > 0 ? C : 1));
    for (int r = r0; r < r1; r++) {
        const uint16_t *xr = x + (size_t)r * C;
        uint16_t *outr = out + (size_t)r * C;
        float rowmax = h2f(xr[0]);
        for (int j = 1; j < C; j++) {
            float v = h2f(xr[j]);
            if (v > rowmax) rowmax = v;
        }
        float rowsum = 0.0f;
        for (int j = 0; j < C; j++) {
            e[j] = expf(h2f(xr[j]) - rowmax);
            rowsum += e[j];
        }
        for (int j = 0; j < C; j++) outr[j] = f2h(e[j] / rowsum);
    }
    free(e);
}

/* kernels/expert/fp16_layernorm/reference.c:9-23 per row, eps parameter */
void oracle_layernorm_f32_rows(const float *x, const float *gamma,
                               const float *beta, float *out, int R, int C,
                               float eps, int r0, int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const float *xr = x + (size_t)r * C;
        float *outr = out + (size_t)r * C;
        float sumx = 0.0f, sumsq = 0.0f;
        for (int i = 0; i < C; i++) {
            float v = xr[i];
            sumx += v;
            sumsq += v * v;
        }
        float mean = sumx / (float)C;
        float var = sumsq / (float)C - mean * mean;
        if (var < 0.0f) var = 0.0f;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < C; i++) {
            float d = (xr[i] - mean) * inv_std;
            outr[i] = d * gamma[i] + beta[i];
        }
    }
}

void oracle_layernorm_f16_rows(const uint16_t *x, const uint16_t *gamma,
                               const uint16_t *beta, uint16_t *out, int R,
                               int C, float eps, int r0, int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const uint16_t *xr = x + (size_t)r * C;
        uint16_t *outr = out + (size_t)r * C;
        float sumx = 0.0f, sumsq = 0.0f;
        for (int i = 0; i < C; i++) {
            float v = h2f(xr[i]);
            sumx += v;
            sumsq += v * v;
        }
        float mean = sumx / (float)C;
        float var = sumsq / (float)C - mean * mean;
        if (var < 0.0f) var = 0.0f;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < C; i++) {
            float d = (h2f(xr[i]) - mean) * inv_std;
            outr[i] = f2h(d * h2f(gamma[i]) + h2f(beta[i]));
        }
    }
}

/* kernels/expert/fp16_rmsnorm/reference.c:7-17 per row, eps parameter */
void oracle_rmsnorm_f32_rows(const float *x, const float *gamma, float *out,
                             int R, int C, float eps, int r0, int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const float *xr = x + (size_t)r * C;
        float *outr = out + (size_t)r * C;
        float sumsq = 0.0f;
        for (int i = 0; i < C; i++) sumsq += xr[i] * xr[i];
        float ms = sumsq / (float)C;
        float inv_rms = 1.0f / sqrtf(ms + eps);
        for (int i = 0; i < C; i++) outr[i] = xr[i] * inv_rms * gamma[i];
    }
}

void oracle_rmsnorm_f16_rows(const uint16_t *x, const uint16_t *gamma,
                             uint16_t *out, int R, int C, float eps, int r0,
                             int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const uint16_t *xr = x + (size_t)r * C;
        uint16_t *outr = out + (size_t)r * C;
        float sumsq = 0.0f;
        for (int i = 0; i < C; i++) {
            float v = h2f(xr[i]);
            sumsq += v * v;
        }
        float ms = sumsq / (float)C;
        float inv_rms = 1.0f / sqrtf(ms + eps);
        for (int i = 0; i < C; i++)
            outr[i] = f2h(h2f(xr[i]) * inv_rms * h2f(gamma[i]));
    }
}

/* kernels/mined/fp32_sum/reference.c:8-14 (acc = acc + x, in order) per
 * row; max seeded at -INFINITY like the mined amax references. */
void oracle_rowreduce_f32_rows(const float *x, float *out, int R, int C,
                               int op, int r0, int r1) {
    (void)R;
    for (int r = r0; r < r1; r++) {
        const float *xr = x + (size_t)r * C;
        float acc;
        if (op == 0) {
            acc = 0.0f;
            for (int j = 0; j < C; j++) acc = acc + xr[j];
        } else {
            acc = -INFINITY;
            for (int j = 0; j < C; j++) acc = xr[j] > acc ? xr[j] : acc;
        }
        out[r] = acc;
    }
}

/* ---- threaded driver ---- */

typedef struct {
    int op;
    const void *args;
    int r0, r1;
} oracle_job;

static void *oracle_job_run(void *p) {
    const oracle_job *j = (const oracle_job *)p;
    switch (j->op) {
    case ORACLE_OP_I8_GEMM_REQUANT: {
        const oracle_gemm_args *a = (const oracle_gemm_args *)j->args;
        oracle_i8_gemm_requant_rows((const int8_t *)a->A, (const int8_t *)a->B,
                                    (int8_t *)a->out, a->M, a->N, a->K, a->mult,
                                    a->shift, (int8_t)a->zp, j->r0, j->r1);
        break;
    }
    case ORACLE_OP_GEMM_U8S8_PC: {
        const oracle_gemm_args *a = (const oracle_gemm_args *)j->args;
        oracle_gemm_u8s8_pc_rows((const uint8_t *)a->A, (const int8_t *)a->B,
                                 a->bias, (uint8_t *)a->out, a->M, a->N, a->K,
                                 a->zpA, a->mult_pc, a->shift_pc,
                                 (uint8_t)a->zp, j->r0, j->r1);
        break;
    }
    case ORACLE_OP_GEMM_F16_NT: {
        const oracle_gemm_args *a = (const oracle_gemm_args *)j->args;
        oracle_gemm_f16_nt_rows((const uint16_t *)a->A, (const uint16_t *)a->B,
                                (uint16_t *)a->out, a->M, a->N, a->K, j->r0, j->r1);
        break;
    }
    case ORACLE_OP_ATTN_F16: {
        /* rows here are (head, query-row) pairs flattened as h * SQ + q */
        const oracle_attn_args *a = (const oracle_attn_args *)j->args;
        size_t qs = (size_t)a->SQ * a->D, ks = (size_t)a->SK * a->D;
        for (int t = j->r0; t < j->r1;) {
            int h = t / a->SQ, q = t % a->SQ;
            int qe = a->SQ;
            if ((h + 1) * a->SQ > j->r1) qe = j->r1 - h * a->SQ;
            oracle_attn_f16_head_rows(a->Q + h * qs, a->K + h * ks, a->V + h * ks,
                                      a->O + h * qs, a->SK, a->D, a->scale,
                                      a->causal, q, qe);
            t = h * a->SQ + qe;
        }
        break;
    }
    case ORACLE_OP_SOFTMAX_F32: {
        const oracle_rows_args *a = (const oracle_rows_args *)j->args;
        oracle_softmax_f32_rows(a->x, a->out, a->R, a->C, j->r0, j->r1);
        break;
    }
    case ORACLE_OP_LAYERNORM_F32: {
        const oracle_rows_args *a = (const oracle_rows_args *)j->args;
        oracle_layernorm_f32_rows(a->x, a->gamma, a->beta, a->out, a->R, a->C,
                                  a->eps, j->r0, j->r1);
        break;
    }
    case ORACLE_OP_ROWREDUCE_F32: {
        const oracle_rows_args *a = (const oracle_rows_args *)j->args;
        oracle_rowreduce_f32_rows(a->x, a->out, a->R, a->C, a->op, j->r0, j->r1);
        break;
    }
    default:
        break;
    }
    return NULL;
}

int oracle_parallel(int op, const void *args, int r0, int r1, int nthreads) {
    if (r1 <= r0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > r1 - r0) nthreads = r1 - r0;
    oracle_job *jobs = (oracle_job *)calloc((size_t)nthreads, sizeof(oracle_job));
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof(pthread_t));
    if (!jobs || !th) {
        free(jobs);
        free(th);
        return -1;
    }
    int n = r1 - r0, rc = 0;
    for (int t = 0; t < nthreads; t++) {
        jobs[t].op = op;
        jobs[t].args = args;
        jobs[t].r0 = r0 + (int)((int64_t)n * t / nthreads);
        jobs[t].r1 = r0 + (int)((int64_t)n * (t + 1) / nthreads);
        if (pthread_create(&th[t], NULL, oracle_job_run, &jobs[t]) != 0) {
            oracle_job_run(&jobs[t]);
            th[t] = 0;
        }
    }
    for (int t = 0; t < nthreads; t++)
        if (th[t]) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    return rc;
}

/* ------------------------------------------------ integer reductions
 * One left-to-right pass per op, as the references:
 *   SUM    vtcm_reduce_i32/reference.c:5-9, i8_sum_dma/reference.c:4-8
 *   SUM64  dma_double_buffer_reduce_i32/reference.c:5-9
 *   SUMSQ  i8_sumsq_i32/reference.c:2-4;  SUMSQ_DIFF i8_sumsq_diff_i32/reference.c:2-9
 *   DOT    i8_weighted_sum/reference.c:2-6;  L1 i8_l1norm_dma/reference.c:6-10
 *   ABSMAX i8_absmax_dma/reference.c:6-13;  MAX dma_stream_max_u8/reference.c:5-9
 *   ARGMAX / ARGMIN i8_argmax_dma/reference.c:6-13, i8_argmin_dma/reference.c:6-13
 *   TOP1   i8_top1_reduce_dma/reference.c:8-16;  MEAN i8_mean_dma/reference.c:6-10
 * The int32 accumulations are done on uint32 (the references' signed int32
 * overflow, defined here as the two's-complement wrap). */
static int64_t red_elem_at(const void *a, int elem, int64_t i) {
    switch (elem) {
    case ORACLE_ELEM_I8: return ((const int8_t *)a)[i];
    case ORACLE_ELEM_U8: return ((const uint8_t *)a)[i];
    case ORACLE_ELEM_I16: return ((const int16_t *)a)[i];
    default: return ((const int32_t *)a)[i];
    }
}

void oracle_reduce_int(const void *a, const void *b, int elem, int64_t n, int op, void *out) {
    int32_t *o32 = (int32_t *)out;
    uint32_t s = 0;
    int64_t s64 = 0;
    if (op == ORACLE_RED_ARGMAX || op == ORACLE_RED_ARGMIN || op == ORACLE_RED_TOP1) {
        int64_t bv = red_elem_at(a, elem, 0), bi = 0;
        for (int64_t i = 1; i < n; i++) {
            const int64_t x = red_elem_at(a, elem, i);
            if (op == ORACLE_RED_ARGMIN ? x < bv : x > bv) {
                bv = x;
                bi = i;
            }
        }
        if (op == ORACLE_RED_TOP1) {
            o32[0] = (int32_t)bv;
            o32[1] = (int32_t)bi;
        } else {
            o32[0] = (int32_t)bi;
        }
        return;
    }
    if (op == ORACLE_RED_MAX || op == ORACLE_RED_MIN || op == ORACLE_RED_ABSMAX) {
        int64_t m = 0;
        for (int64_t i = 0; i < n; i++) {
            int64_t x = red_elem_at(a, elem, i);
            if (op == ORACLE_RED_ABSMAX) x = x < 0 ? -x : x;
            if (i == 0 && op != ORACLE_RED_ABSMAX) m = x;
            else if (op == ORACLE_RED_MIN ? x < m : x > m) m = x;
        }
        o32[0] = (int32_t)m;
        return;
    }
    for (int64_t i = 0; i < n; i++) {
        const int64_t x = red_elem_at(a, elem, i);
        const int64_t y = (op == ORACLE_RED_SUMSQ_DIFF || op == ORACLE_RED_DOT)
                              ? red_elem_at(b, elem, i) : 0;
        switch (op) {
        case ORACLE_RED_SUM64: s64 += x; break;
        case ORACLE_RED_SUMSQ: s += (uint32_t)x * (uint32_t)x; break;
        case ORACLE_RED_SUMSQ_DIFF: {
            const uint32_t d = (uint32_t)(x - y);
            s += d * d;
            break;
        }
        case ORACLE_RED_DOT: s += (uint32_t)x * (uint32_t)y; break;
        case ORACLE_RED_L1: s += (uint32_t)(x < 0 ? -x : x); break;
        default: s += (uint32_t)x; break;   /* SUM, MEAN */
        }
    }
    if (op == ORACLE_RED_SUM64) *(int64_t *)out = s64;
    else if (op == ORACLE_RED_MEAN) o32[0] = (int32_t)((int64_t)(int32_t)s / n);
    else o32[0] = (int32_t)s;
}

/* hvx_vmax_i8/reference.c:3-6, hvx_vmax_u8/reference.c:3-6,
 * hvx_vmin_i16/reference.c:3-6, hvx_vmin_u8/reference.c:3-6,
 * i8_max_scalar_dma/reference.c:6-11, i8_min_scalar_dma/reference.c:6-11 */
void oracle_minmax_ew(const void *a, const void *b, int32_t c, int elem, int op, void *out,
                      int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const int64_t x = red_elem_at(a, elem, i);
        int64_t y = b ? red_elem_at(b, elem, i) : 0;
        if (!b) {   /* the scalar in the element's own type */
            if (elem == ORACLE_ELEM_I8) y = (int8_t)c;
            else if (elem == ORACLE_ELEM_U8) y = (uint8_t)c;
            else y = (int16_t)c;
        }
        const int64_t r = op ? (x < y ? x : y) : (x > y ? x : y);
        if (elem == ORACLE_ELEM_I16) ((int16_t *)out)[i] = (int16_t)r;
        else ((uint8_t *)out)[i] = (uint8_t)r;
    }
}

/* hvx_vradd_i8_reduce/reference.c:3-10 with the group width a parameter */
void oracle_group_sum_i8(const int8_t *a, int32_t *out, int64_t g, int w) {
    for (int64_t k = 0; k < g; k++) {
        uint32_t s = 0;
        for (int j = 0; j < w; j++) s += (uint32_t)(int32_t)a[k * w + j];
        out[k] = (int32_t)s;
    }
}

/* hvx_vrmpy_i8_dot/reference.c:3-9 (w = 4) */
void oracle_group_dot_i8(const int8_t *a, const int8_t *b, int32_t *out, int64_t g, int w) {
    for (int64_t k = 0; k < g; k++) {
        uint32_t s = 0;
        for (int j = 0; j < w; j++) s += (uint32_t)((int32_t)a[k * w + j] * (int32_t)b[k * w + j]);
        out[k] = (int32_t)s;
    }
}

/* mlp_gate_silu_i8/reference.c:4-15 */
void oracle_gate_mul_requant_i8(const int8_t *gate, const int8_t *up, const int8_t *lut,
                                int8_t *out, int64_t n, int32_t mult, int shift) {
    for (int64_t i = 0; i < n; i++) {
        const int32_t g = lut[(uint8_t)((int)gate[i] + 128)];
        const int64_t q = rq_round((int64_t)(g * (int32_t)up[i]) * (int64_t)mult, shift);
        out[i] = (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
    }
}

/* i8_scan_max/reference.c:2-8 */
void oracle_scan_max_i8(const int8_t *in, int8_t *out, int64_t n) {
    int8_t cur = -128;
    for (int64_t i = 0; i < n; i++) {
        if (in[i] > cur) cur = in[i];
        out[i] = cur;
    }
}

/* gqa_group_reduce_i8/reference.c:6-26 */
void oracle_head_group_reduce_i8(const int8_t *X, int8_t *Y, int H, int G, int64_t MN,
                                 int32_t mult, int shift) {
    const int hpg = H / G;
    for (int g = 0; g < G; g++)
        for (int64_t i = 0; i < MN; i++) {
            int32_t acc = 0;
            for (int t = 0; t < hpg; t++) acc += X[(int64_t)(g * hpg + t) * MN + i];
            int64_t q = rq_round((int64_t)acc * (int64_t)mult, shift);
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            Y[(int64_t)g * MN + i] = (int8_t)q;
        }
}

/* ---------------------------------- integer rows with the table arithmetic */
static int32_t sat8i(int32_t v) { return v > 127 ? 127 : (v < -128 ? -128 : v); }

/* i8_layernorm_dma/reference.c:4-28 (layernorm_row), i8_instance_norm/
 * reference.c:4-40 (per channel: gamma[c], beta[c], table inv_lut + 256 c),
 * i8_chunk_norm/reference.c:4-38 (chunk c: gamma + c chunk), layernorm_residual/
 * reference.c:4-40 (saturating residual add first), embedding_layer_norm/
 * reference.c:4-35 (rows gathered by idx) */
void oracle_layernorm_lut_i8(const int8_t *x, const int32_t *idx, const int8_t *res, int8_t *out,
                             int R, int W, const int8_t *gamma, const int8_t *beta,
                             const uint8_t *inv_lut, int affine) {
    int32_t *t = (int32_t *)malloc(sizeof(int32_t) * (size_t)W);
    for (int r = 0; r < R; r++) {
        const int8_t *xr = x + (size_t)(idx ? idx[r] : r) * W;
        for (int j = 0; j < W; j++) t[j] = res ? sat8i((int32_t)xr[j] + res[(size_t)r * W + j]) : xr[j];
        uint32_t sum = 0;
        for (int j = 0; j < W; j++) sum += (uint32_t)t[j];
        /* affine 3: rmsnorm_residual/reference.c:4-36, mean 0 and no beta */
        const int32_t mu = affine == 3 ? 0 : (int32_t)sum / W;
        uint32_t vs = 0;
        for (int j = 0; j < W; j++) {
            const int32_t d = t[j] - mu;
            vs += (uint32_t)(d * d);
        }
        const int32_t var = (int32_t)vs / W;
        const int vi = var < 0 ? 0 : (var > 255 ? 255 : var);
        const int32_t inv = (affine == 2 ? inv_lut + 256 * (size_t)r : inv_lut)[vi];
        for (int j = 0; j < W; j++) {
            const size_t gj = affine == 1 ? (size_t)r * W + j : (size_t)j;
            const int32_t g = affine == 2 ? gamma[r] : gamma[gj];
            const int32_t b = affine == 3 ? 0 : (affine == 2 ? beta[r] : beta[gj]);
            const int32_t d = t[j] - mu;
            const int32_t scaled = (d * g + 64) >> 7;
            const int32_t normed = (scaled * inv + 128) >> 8;
            out[(size_t)r * W + j] = (int8_t)sat8i(normed + b);
        }
    }
    free(t);
}

/* layernorm_row_i16/reference.c:6-35, layernorm_affine_i16/reference.c:6-37 */
void oracle_layernorm_lut_i16(const int16_t *x, int16_t *out, int R, int C, const int16_t *gamma,
                              const int16_t *beta, const uint16_t *inv_lut, int order) {
    for (int r = 0; r < R; r++) {
        const int16_t *xr = x + (size_t)r * C;
        int64_t sum = 0;
        for (int c = 0; c < C; c++) sum += xr[c];
        const int32_t mu = (int32_t)(sum / C);
        int64_t vs = 0;
        for (int c = 0; c < C; c++) {
            const int64_t d = (int64_t)xr[c] - mu;
            vs += d * d;
        }
        int32_t vi = (int32_t)((vs / C) >> 5);
        vi = vi < 0 ? 0 : (vi > 255 ? 255 : vi);
        const int32_t inv = inv_lut[vi];
        for (int c = 0; c < C; c++) {
            const int32_t d = (int32_t)xr[c] - mu;
            int32_t v;
            if (order == 0) {
                const int32_t scaled = (d * (int32_t)gamma[c] + 32) >> 6;
                v = ((scaled * inv + 512) >> 10) + beta[c];
            } else {
                const int32_t normed = (d * inv + 512) >> 10;
                v = ((normed * (int32_t)gamma[r] + 32) >> 6) + beta[r];
            }
            out[(size_t)r * C + c] = (int16_t)(v > 32767 ? 32767 : (v < -32768 ? -32768 : v));
        }
    }
}

/* i8_gemm_softmax_tile/reference.c:28-48, softmax_rowwise/reference.c:4-27;
 * with recip_lut softmax_row_i8/reference.c:4-33 */
void oracle_lut_softmax_u8(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut,
                           const uint16_t *recip_lut) {
    for (int r = 0; r < R; r++) {
        const int8_t *row = x + (size_t)r * C;
        int8_t m = row[0];
        for (int j = 1; j < C; j++) if (row[j] > m) m = row[j];
        int32_t S = 0;
        for (int j = 0; j < C; j++) {
            int diff = (int)row[j] - (int)m;
            if (diff < -255) diff = -255;
            S += exp_lut[diff + 255];
        }
        const int32_t half = S / 2;
        int32_t sidx = S >> 6;
        if (sidx < 0) sidx = 0;
        if (sidx > 255) sidx = 255;
        const int32_t recip = recip_lut ? recip_lut[sidx] : 0;
        for (int j = 0; j < C; j++) {
            int diff = (int)row[j] - (int)m;
            if (diff < -255) diff = -255;
            const int32_t e = exp_lut[diff + 255];
            if (recip_lut) {
                int32_t v = (e * recip + 32768) >> 16;
                out[(size_t)r * C + j] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
            } else {
                out[(size_t)r * C + j] = (uint8_t)(S > 0 ? (e * 255 + half) / S : 0);
            }
        }
    }
}

/* vtcm_softmax_row_i16/reference.c:6-30 */
void oracle_lut_softmax_i16(const int16_t *x, int16_t *out, int R, int C, const uint16_t *exp_lut) {
    for (int r = 0; r < R; r++) {
        const int16_t *row = x + (size_t)r * C;
        int16_t m = row[0];
        for (int j = 1; j < C; j++) if (row[j] > m) m = row[j];
        int64_t S = 0;
        for (int j = 0; j < C; j++) {
            int32_t diff = (int32_t)row[j] - (int32_t)m;
            if (diff < -255) diff = -255;
            S += exp_lut[diff + 255];
        }
        const int64_t half = S / 2;
        for (int j = 0; j < C; j++) {
            int32_t diff = (int32_t)row[j] - (int32_t)m;
            if (diff < -255) diff = -255;
            out[(size_t)r * C + j] = (int16_t)(S > 0 ? ((int64_t)exp_lut[diff + 255] * 32767 + half) / S : 0);
        }
    }
}

/* attention_scale_i16/reference.c:4-16 */
void oracle_requant_i16(const int32_t *a, int16_t *out, int64_t n, int32_t mult, int shift) {
    for (int64_t i = 0; i < n; i++) {
        const int64_t q = rq_round((int64_t)a[i] * (int64_t)mult, shift);
        out[i] = (int16_t)(q > 32767 ? 32767 : (q < -32768 ? -32768 : q));
    }
}

/* i8_norm_requant_dma/reference.c:11-32 */
void oracle_norm_requant_i8(const int8_t *a, int8_t *out, int64_t n, int nch, const int32_t *nmult,
                            const int *nshift, int32_t mult, int shift, int zp) {
    const int64_t per = n / nch;
    for (int c = 0; c < nch; c++)
        for (int64_t i = 0; i < per; i++) {
            const int64_t v = rq_round((int64_t)a[c * per + i] * nmult[c], nshift[c]);
            const int64_t r = rq_round(v * (int64_t)mult, shift) + zp;
            out[c * per + i] = (int8_t)(r > 127 ? 127 : (r < -128 ? -128 : r));
        }
}

/* rmsnorm_gain_fp16/reference.c:4-19 */
void oracle_rmsnorm_gain_f16(const uint16_t *x, const uint16_t *gain, uint16_t *out, int R, int C,
                             float eps) {
    for (int r = 0; r < R; r++) {
        const uint16_t *xr = x + (size_t)r * C;
        float sumsq = 0.0f;
        for (int c = 0; c < C; c++) {
            const float v = h2f(xr[c]);
            sumsq += v * v;
        }
        const float ms = sumsq / (float)C;
        const float inv_rms = 1.0f / sqrtf(ms + eps);
        const float g = h2f(gain[r]);
        for (int c = 0; c < C; c++) out[(size_t)r * C + c] = f2h(h2f(xr[c]) * inv_rms * g);
    }
}

/* kv_cache_update/reference.c:14-25 */
void oracle_kv_cache_update_i8(int8_t *k_cache, int8_t *v_cache, const int8_t *k_new,
                               const int8_t *v_new, int pos, int heads, int cache_len,
                               int head_dim) {
    for (int h = 0; h < heads; h++) {
        const size_t base = ((size_t)h * cache_len + pos) * head_dim;
        for (int d = 0; d < head_dim; d++) {
            k_cache[base + d] = k_new[(size_t)h * head_dim + d];
            v_cache[base + d] = v_new[(size_t)h * head_dim + d];
        }
    }
}

/* rope_pair_fp16/reference.c:5-13 (built with -ffp-contract=off: each
 * product and sum is rounded to fp32) */
void oracle_rope_pair_f16(const uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                          uint16_t *out, int64_t n_pairs) {
    for (int64_t p = 0; p < n_pairs; p++) {
        const float xr = h2f(x[2 * p]), xi = h2f(x[2 * p + 1]);
        const float c = h2f(cos_t[p]), s = h2f(sin_t[p]);
        out[2 * p] = f2h(xr * c - xi * s);
        out[2 * p + 1] = f2h(xr * s + xi * c);
    }
}

/* i8_ffn_block/reference.c:8-27 (FFN_SH1 / FFN_SH2 as sh1 / sh2) */
void oracle_ffn_hmx_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2,
                       const int32_t *b2, int8_t *out, int M, int D, int Dff, int sh1, int sh2) {
    int8_t *H = (int8_t *)malloc((size_t)M * (Dff > 0 ? Dff : 1));
    for (int i = 0; i < M; i++)
        for (int j = 0; j < Dff; j++) {
            int acc = 0;
            for (int k = 0; k < D; k++) acc += (int)X[(size_t)i * D + k] * (int)W1[(size_t)k * Dff + j];
            const int p1 = sx12(hmx_field_i(acc)) + b1[j];
            int h = p1 > 0 ? (p1 >> sh1) : 0;
            H[(size_t)i * Dff + j] = (int8_t)(h > 127 ? 127 : h);
        }
    for (int i = 0; i < M; i++)
        for (int j = 0; j < D; j++) {
            int acc = 0;
            for (int k = 0; k < Dff; k++) acc += (int)H[(size_t)i * Dff + k] * (int)W2[(size_t)k * D + j];
            out[(size_t)i * D + j] = (int8_t)clamp_i8i((sx12(hmx_field_i(acc)) + b2[j]) >> sh2);
        }
    free(H);
}

/* i8_ffn_swiglu_block/reference.c:10-34 with kernel_api.h's sw_scale,
 * sw_gate and sw_hu (SW_SG, SW_SU, SW_SH, SW_ZP, SW_SO as sg, su, sh, zp, so) */
void oracle_ffn_swiglu_hmx_i8(const uint8_t *X, const int8_t *Wg, const int8_t *Wu,
                              const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut,
                              int8_t *out, int M, int D, int Dff, int sg, int su, int sh, int zp,
                              int so) {
    uint8_t *Hu = (uint8_t *)malloc((size_t)M * (Dff > 0 ? Dff : 1));
    for (int i = 0; i < M; i++)
        for (int j = 0; j < Dff; j++) {
            int gacc = 0, uacc = 0;
            for (int k = 0; k < D; k++) {
                gacc += (int)X[(size_t)i * D + k] * (int)Wg[(size_t)k * Dff + j];
                uacc += (int)X[(size_t)i * D + k] * (int)Wu[(size_t)k * Dff + j];
            }
            const int gq = clamp_i8i(sx12(hmx_field_i(gacc)) >> sg);
            const int uq = clamp_i8i(sx12(hmx_field_i(uacc)) >> su);
            const int silu_g = (signed char)silu_lut[gq + 128];
            int h = (silu_g * uq) >> sh;
            if (h > zp - 1) h = zp - 1;
            if (h < -zp) h = -zp;
            Hu[(size_t)i * Dff + j] = (uint8_t)(h + zp);
        }
    for (int i = 0; i < M; i++)
        for (int m = 0; m < D; m++) {
            int acc = 0;
            for (int j = 0; j < Dff; j++) acc += (int)Hu[(size_t)i * Dff + j] * (int)Wd[(size_t)j * D + m];
            out[(size_t)i * D + m] = (int8_t)clamp_i8i((sx12(hmx_field_i(acc)) + bd[m]) >> so);
        }
    free(Hu);
}

/* i8_transformer_encoder_block/reference.c:18-78 (ATTN_SCALE_SHIFT 4,
 * ATTN_OUT_SHIFT 8, FFN_SH1 8, FFN_SH2 4) */
void oracle_encoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut,
                             int8_t *out, int S, int D, int Dff) {
    int8_t *sc = (int8_t *)malloc((size_t)S * S);
    uint8_t *pr = (uint8_t *)malloc((size_t)S * S);
    uint8_t *h = (uint8_t *)malloc((size_t)S * D);
    uint8_t *Hb = (uint8_t *)malloc((size_t)S * (Dff > 0 ? Dff : 1));
    for (int i = 0; i < S; i++)
        for (int j = 0; j < S; j++) {
            int acc = 0;
            for (int d = 0; d < D; d++) acc += (int)X[(size_t)i * D + d] * (int)(int8_t)X[(size_t)j * D + d];
            sc[(size_t)i * S + j] = (int8_t)clamp_i8i(sx12(hmx_field_i(acc)) >> 4);
        }
    for (int i = 0; i < S; i++) lut_softmax_row(sc + (size_t)i * S, pr + (size_t)i * S, S, S, exp_lut);
    for (int i = 0; i < S; i++)
        for (int d = 0; d < D; d++) {
            int acc = 0;
            for (int j = 0; j < S; j++) acc += (int)pr[(size_t)i * S + j] * (int)(int8_t)X[(size_t)j * D + d];
            const int a = clamp_i8i(sx12(hmx_field_i(acc)) >> 8);
            h[(size_t)i * D + d] = (uint8_t)clamp_u8i((int)X[(size_t)i * D + d] + a);
        }
    for (int i = 0; i < S; i++)
        for (int j = 0; j < Dff; j++) {
            int acc = 0;
            for (int k = 0; k < D; k++) acc += (int)h[(size_t)i * D + k] * (int)W1[(size_t)k * Dff + j];
            const int p1 = sx12(hmx_field_i(acc)) + b1[j];
            const int hh = p1 > 0 ? (p1 >> 8) : 0;
            Hb[(size_t)i * Dff + j] = (uint8_t)(hh > 127 ? 127 : hh);
        }
    for (int i = 0; i < S; i++)
        for (int j = 0; j < D; j++) {
            int acc = 0;
            for (int k = 0; k < Dff; k++) acc += (int)Hb[(size_t)i * Dff + k] * (int)W2[(size_t)k * D + j];
            const int fv = (sx12(hmx_field_i(acc)) + b2[j]) >> 4;
            out[(size_t)i * D + j] = (int8_t)clamp_i8i((int)h[(size_t)i * D + j] + fv);
        }
    free(sc); free(pr); free(h); free(Hb);
}

/* rescale_i16_i8_dma/reference.c:5-15, dequant_i8_i16_dma/reference.c:5-12,
 * hmx_requant_store_i8/reference.c:3-8, i8_add_bias_sat_dma/reference.c:3-9,
 * i8_element_affine_dma/reference.c:5-16: one affine form with their
 * int32 (wrap32) or int64 arithmetic and their rounding */
void oracle_affine_ew(const void *in, int elem_in, void *out, int elem_out, int64_t n, int32_t zp_in,
                      int32_t mult, int64_t add, int shift, int round, int wrap32, int zp_out,
                      int32_t lo, int32_t hi) {
    for (int64_t i = 0; i < n; i++) {
        int64_t x;
        switch (elem_in) {
        case 0: x = ((const int8_t *)in)[i]; break;
        case 1: x = ((const uint8_t *)in)[i]; break;
        case 2: x = ((const int16_t *)in)[i]; break;
        default: x = ((const int32_t *)in)[i]; break;
        }
        int64_t v = wrap32 ? (int64_t)(int32_t)(((uint32_t)(int32_t)x - (uint32_t)zp_in) * (uint32_t)mult +
                                                (uint32_t)add)
                           : (x - zp_in) * (int64_t)mult + add;
        int64_t r = round ? (v >> shift) : rq_round(v, shift);
        r += zp_out;
        if (r < lo) r = lo;
        if (r > hi) r = hi;
        switch (elem_out) {
        case 0: ((int8_t *)out)[i] = (int8_t)r; break;
        case 1: ((uint8_t *)out)[i] = (uint8_t)r; break;
        case 2: ((int16_t *)out)[i] = (int16_t)r; break;
        default: ((int32_t *)out)[i] = (int32_t)r; break;
        }
    }
}

/* i16_gemm/reference.c:2-11 (int32 accumulator, modulo 2^32) */
void oracle_gemm_i16(const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K) {
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            uint32_t acc = 0;
            for (int k = 0; k < K; k++)
                acc += (uint32_t)((int32_t)A[(size_t)i * K + k] * (int32_t)B[(size_t)k * N + j]);
            C[(size_t)i * N + j] = (int32_t)acc;
        }
}

static int8_t rq_biased_i8(int32_t acc, int32_t bias, int32_t mult, int shift, int zp) {
    return sat_i8(rq_round(((int64_t)acc + bias) * (int64_t)mult, shift) + zp);
}

/* i8_channel_mix_block/reference.c:17-40 (TOKENS x CHANNELS as M x K,
 * D_FF as V, CHANNELS out as D; lut NULL: no table) */
void oracle_mix_mlp_i8(const int8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *lut,
                       const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V, int D,
                       int32_t mult1, int shift1, int32_t mult2, int shift2) {
    int8_t *y = (int8_t *)malloc((size_t)(V > 0 ? V : 1));
    for (int t = 0; t < M; t++) {
        for (int m = 0; m < V; m++) {
            uint32_t acc = 0;
            for (int c = 0; c < K; c++) acc += (uint32_t)((int32_t)W1[(size_t)m * K + c] * X[(size_t)t * K + c]);
            const int8_t q = rq_biased_i8((int32_t)acc, b1[m], mult1, shift1, 0);
            y[m] = lut ? lut[(uint8_t)((int)q + 128)] : q;
        }
        for (int c = 0; c < D; c++) {
            uint32_t acc = 0;
            for (int m = 0; m < V; m++) acc += (uint32_t)((int32_t)W2[(size_t)c * V + m] * y[m]);
            out[(size_t)t * D + c] = rq_biased_i8((int32_t)acc, b2[c], mult2, shift2, 0);
        }
    }
    free(y);
}

/* i8_token_mix_block/reference.c:17-41 */
void oracle_token_mix_i8(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2,
                         const int32_t *b2, int8_t *out, int T, int C, int DM, int32_t mult1,
                         int shift1, int32_t mult2, int shift2) {
    int8_t *y = (int8_t *)malloc((size_t)(DM > 0 ? DM : 1));
    for (int c = 0; c < C; c++) {
        for (int m = 0; m < DM; m++) {
            uint32_t acc = 0;
            for (int t = 0; t < T; t++) acc += (uint32_t)((int32_t)W[(size_t)m * T + t] * X[(size_t)t * C + c]);
            y[m] = rq_biased_i8((int32_t)acc, b[m], mult1, shift1, 0);
        }
        for (int t = 0; t < T; t++) {
            uint32_t acc = 0;
            for (int m = 0; m < DM; m++) acc += (uint32_t)((int32_t)W2[(size_t)t * DM + m] * y[m]);
            out[(size_t)t * C + c] = rq_biased_i8((int32_t)acc, b2[t], mult2, shift2, 0);
        }
    }
    free(y);
}

/* rnn_cell_i8/reference.c: acc = b + Wx x + Wh h (int32), requant + zp,
 * saturate, h_t = tanh_lut[(uint8) pre_act] */
void oracle_rnn_cell_i8(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x,
                        const int8_t *h_prev, int8_t *h_t, int H, int I, int32_t mult, int shift,
                        int zp, const int8_t *tanh_lut) {
    for (int j = 0; j < H; j++) {
        uint32_t acc = (uint32_t)b[j];
        for (int k = 0; k < I; k++) acc += (uint32_t)((int32_t)Wx[(size_t)j * I + k] * x[k]);
        for (int k = 0; k < H; k++) acc += (uint32_t)((int32_t)Wh[(size_t)j * H + k] * h_prev[k]);
        const int8_t pre = sat_i8(rq_round((int64_t)(int32_t)acc * (int64_t)mult, shift) + zp);
        h_t[j] = tanh_lut[(uint8_t)pre];
    }
}

/* i8_conv2d_3x3_hmx/reference.c, i8_conv2d_3x3_hmx_tiled/reference.c,
 * i8_conv2d_bias_relu_hmx/reference.c, i8_conv1d_bias_requant_hmx/reference.c:
 * window sums, the 12-bit HMX field, bias, activation, store (store /
 * act numbered as ORACLE_HMX_STORE_* / ORACLE_HMX_ACT_*) */
void oracle_conv2d_hmx(const uint8_t *in, const int8_t *W, const int32_t *bias, void *out, int store,
                       int act, int c_in, int ih, int iw, int c_out, int kh, int kw, int stride) {
    const int oh = (ih - kh) / stride + 1, ow = (iw - kw) / stride + 1;
    for (int co = 0; co < c_out; co++)
        for (int y = 0; y < oh; y++)
            for (int x = 0; x < ow; x++) {
                int acc = 0;
                for (int ci = 0; ci < c_in; ci++)
                    for (int a = 0; a < kh; a++)
                        for (int b = 0; b < kw; b++)
                            acc += (int)in[((size_t)ci * ih + y * stride + a) * iw + x * stride + b] *
                                   (int)W[(((size_t)co * c_in + ci) * kh + a) * kw + b];
                const int f = hmx_field_i(acc);
                int v = sx12(f) + (bias ? bias[co] : 0);
                if (act == ORACLE_HMX_ACT_RELU && v < 0) v = 0;
                const size_t o = ((size_t)co * oh + y) * ow + x;
                if (store == ORACLE_HMX_STORE_U16_FIELD)
                    ((uint16_t *)out)[o] = (uint16_t)(v & 0xFFF);
                else if (store == ORACLE_HMX_STORE_I8_SAT)
                    ((int8_t *)out)[o] = (int8_t)clamp_i8i(v);
                else
                    ((int32_t *)out)[o] = v;
            }
}
