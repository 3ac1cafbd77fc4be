/* hexoracle.h -- CPU oracle for the hot-path operators (TEST INFRASTRUCTURE).
 *
 * This library is the checker, never the product: only tests/, the smoke()
 * entry of __graft_entry__.py and the cpu_baseline / --impl reference legs of
 * bench.py may load it.  The CUDA path in hexkernels_b200/ never calls it.
 *
 * Every function restates one scalar reference.c of the hexkernels corpus
 * (sriharshapy/hexkernels, paths relative to that repository) with the same
 * arithmetic, the same summation order and the same rounding; the restatement
 * only lifts fixed-size stack arrays and adds row ranges [r0, r1) so a caller
 * can split the rows across threads.  Parity is pinned by tests/golden/, whose
 * expected outputs were produced by the reference's own reference.c files
 * compiled here (oracle/Makefile target `ref`, script tests/golden/make_golden.py).
 *
 * fp16 values travel as uint16_t bit patterns (IEEE binary16); the C side
 * converts with _Float16, which rounds to nearest-even like the reference's
 * __fp16 casts.
 */
#ifndef HEXORACLE_H
#define HEXORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- integer GEMM + fixed-point requant family ---- */

/* kernels/expert/i8_gemm_requant/reference.c:2-20 */
void oracle_i8_gemm_requant_rows(const int8_t *A, const int8_t *B, int8_t *out,
                                 int M, int N, int K, int32_t mult, int shift,
                                 int8_t zp, int r0, int r1);

/* kernels/expert/i8_gemm_bias_requant/reference.c:2-24 */
void oracle_i8_gemm_bias_requant_rows(const int8_t *A, const int8_t *B,
                                      const int32_t *bias, int8_t *out,
                                      int M, int N, int K, int32_t mult,
                                      int shift, int8_t zp, int r0, int r1);

/* kernels/expert/gemm_tile_zp_i8/reference.c:6-30 */
void oracle_gemm_tile_zp_i8_rows(const int8_t *A, const int8_t *B, int8_t *out,
                                 int M, int N, int K, int32_t zpA,
                                 int32_t scale_mult, int scale_shift,
                                 int r0, int r1);

/* Composed u8 x s8 asymmetric GEMM with per-output-channel requant to u8:
 * zero-point decomposition of gemm_tile_zp_i8/reference.c:10-19, bias add of
 * i8_gemm_bias_requant/reference.c:13, per-channel (column j) mult/shift of
 * requant_per_channel/reference.c:5-10, u8 saturation with zp of
 * requantize_i32_u8_dma/reference.c:5-13. */
void oracle_gemm_u8s8_pc_rows(const uint8_t *A, const int8_t *B,
                              const int32_t *bias, uint8_t *out,
                              int M, int N, int K, int32_t zpA,
                              const int32_t *mult, const int *shift,
                              uint8_t zp_out, int r0, int r1);

/* HMX-convention int8 GEMMs: acc = sum_k (A[i][k] - zpA) * B[k][j] (int32),
 * r = sx12((acc * 17 + 8) >> 4) (the matrix engine's 0x40-config requant
 * field, sign-extended from 12 bits), then by `mode`:
 *   0: out int32 = r   (hmx_matmul_i8_64/reference.c:4-12,
 *                       hmx_matmul_i8_deepk/reference.c:10-17,
 *                       hmx_matmul_i8_zp/reference.c:14-22,
 *                       hmx_matmul_i8_transposeB/reference.c:13-21)
 *   1: out int8 = clamp(r, -128, 127)   (hmx_matmul_i8_requant/reference.c:4-13)
 *   2: out uint8 = clamp(max(r + bias[j], 0), 0, 255)
 *                       (i8_gemm_bias_relu_requant_hmx/reference.c:20-31)
 * A uint8 [M][K]; B int8 [K][N], or Bt [N][K] when b_transposed. */
void oracle_gemm_hmx_rows(const uint8_t *A, const int8_t *B, int b_transposed,
                          const int32_t *bias, void *out, int M, int N, int K,
                          int32_t zpA, int mode, int r0, int r1);

/* General form of the HMX-convention family: v = sx12((acc * 17 + 8) >> 4),
 * then v += bias[j] (if bias), v += res[i][j] (int32 or int8 [M][N] residual),
 * the activation, and the store:
 *   I32 v; I8_SAT clamp(v,-128,127); U8_SAT clamp(v,0,255); I8_LOW (int8)(v & 0xFF);
 *   U16_FIELD v & 0xFFF; LUT_I32 lut32[clamp(v+128,0,255)];
 *   LUT_I8 lut8[(uint8)(sat_i8(v)+128)]
 * activation RELU max(v,0), LEAKY_SHR3 v >= 0 ? v : v >> 3.  col_major stores
 * out[j*M + i].  References (kernels/expert/<bundle>/reference.c):
 *   hmx_matmul_i8_32, _accum_chain, _multi_n, _rect_32x64, hmx_kacc_i8_2tile,
 *   _4tile, hmx_tile_mac_i8_32, hmx_gemv_i8 (I32); hmx_matmul_i8_bias,
 *   i8_matmul_bias_hmx (I32 + bias); hmx_matmul_i8_bias_relu,
 *   i8_matmul_bias_relu_hmx (+ RELU); hmx_matmul_i8_relu, i8_gemm_relu_hmx_deepk
 *   (RELU); i8_matmul_leaky_relu_hmx (LEAKY_SHR3); hmx_matmul_i8_col_major
 *   (col_major); hmx_matmul_i8_gelu_lut (LUT_I32); i8_matmul_hmx_64x64, _96x96
 *   (U16_FIELD, hvx_hmx_requant_0x40 of env/harness/harness_common.h:127);
 *   i8_matmul_hmx_requant (I8_LOW); i8_matmul_residual_hmx (RES_I32);
 *   i8_matmul_add_requant_hmx (RES_I8, I8_SAT); i8_matmul_bias_gelu_hmx
 *   (bias, LUT_I8); i8_linear_proj_hmx (Bt, bias, I8_SAT). */
enum {
    ORACLE_HMX_STORE_I32 = 0, ORACLE_HMX_STORE_I8_SAT = 1, ORACLE_HMX_STORE_U8_SAT = 2,
    ORACLE_HMX_STORE_I8_LOW = 3, ORACLE_HMX_STORE_U16_FIELD = 4, ORACLE_HMX_STORE_LUT_I32 = 5,
    ORACLE_HMX_STORE_LUT_I8 = 6, ORACLE_HMX_STORE_ACC_I32 = 7,
    ORACLE_HMX_ACT_NONE = 0, ORACLE_HMX_ACT_RELU = 1, ORACLE_HMX_ACT_LEAKY_SHR3 = 2,
    ORACLE_HMX_RES_NONE = 0, ORACLE_HMX_RES_I32 = 1, ORACLE_HMX_RES_I8 = 2,
};
void oracle_gemm_hmx_ex_rows(const uint8_t *A, const int8_t *B, int b_transposed,
                             void *out, int M, int N, int K, int32_t zpA, int store,
                             int act, const int32_t *bias, int res_kind, const void *res,
                             const void *lut, int col_major, int r0, int r1);

/* kernels/expert/i8_attention_qkt_av_hmx/reference.c: Sc = sx12 field of
 * Q K^T (Q [SQ][D] u8, K [SK][D] s8), out [SQ][D] = sx12 field of Sc V
 * (V [SK][D] s8); int accumulation with wrap. */
void oracle_attn_qkt_av_hmx(const uint8_t *Q, const int8_t *K, const int8_t *V, int32_t *out,
                            int SQ, int SK, int D);

/* int8 LUT-softmax attention, per query head hq (KV head hq / (HQ / HKV)):
 *   mode 0  kernels/expert/gqa_attention/reference.c (Q int8, out int8)
 *   mode 1  i8_attention_block/reference.c, i8_gqa_attention_block/reference.c
 *           (Q u8, out uint16)
 *   mode 2  i8_rope_attention_block/reference.c (mode 1 after the rotation)
 * Q [HQ][S][D], K / V [HKV][S][D], out [HQ][S][D]. */
void oracle_attn_lut_i8(int mode, const void *Q, const int8_t *K, const int8_t *V,
                        const uint8_t *exp_lut, const int8_t *cos_lut, const int8_t *sin_lut,
                        int rot_shift, void *out, int HQ, int HKV, int S, int D,
                        int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift);
/* mode 0 with the banded mask of kernels/expert/i8_sparse_attn_block/
 * reference.c: scores with |i - j| > window are -128 (still in the softmax). */
void oracle_attn_lut_i8_window(const int8_t *Q, const int8_t *K, const int8_t *V,
                               const uint8_t *exp_lut, int8_t *out, int heads, int S, int D, int window,
                               int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift);
/* kernels/expert/i8_decoder_block/reference.c */
void oracle_decoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                             const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff);

/* s8 x s8 GEMM + requant with optional bias and a ReLU between bias add and
 * requant (kernels/expert/gemm_bias_relu_requant/reference.c; the matrix-
 * vector i8_linear_relu_requant / i8_matvec_bias_requant as A = x, Bt = matrix). */
void oracle_gemm_i8_rq_ex_rows(const int8_t *A, const int8_t *B, int b_transposed,
                               const int32_t *bias, const int8_t *res, int8_t *out, int M, int N,
                               int K, int32_t mult, int shift, int zp, int relu, int r0, int r1);
/* s8 (a_signed) / u8 A x s8 B on the raw int32 accumulator, int64 post-ops:
 * x = acc + bias[j] + res[i][j]; activation; store (ORACLE_HMX_STORE_*).
 * kernels/expert/{gemm_tile_i8,gemm_tile_deepk_i8,i8_gemm_tile,i8_gemm_bias,
 * gemm_tile_bias_relu_i8,gemm_bias_gelu,i8_gemm_gelu_lut,ffn_up_gelu_i8}/reference.c */
void oracle_gemm_i8_acc_rows(const void *A, int a_signed, const int8_t *B, int b_transposed,
                             const int32_t *bias, const void *res, int res_kind, const void *lut,
                             void *out, int store, int act, int M, int N, int K, int r0, int r1);
/* kernels/expert/ffn_relu_block/reference.c: two GEMM layers, ReLU + sat8
 * between, requant after. */
void oracle_ffn_relu_i8(const int8_t *A, const int8_t *W1, const int32_t *b1, const int8_t *W2,
                        const int32_t *b2, int8_t *out, int M, int K, int V, int D, int32_t mult,
                        int shift, int zp);
/* kernels/expert/mlp_block/reference.c: the first layer's activation is
 * act_lut[sat8(acc + b1) + 128]. */
void oracle_ffn_lut_i8(const int8_t *A, const int8_t *W1, const int32_t *b1, const int8_t *act_lut,
                       const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V, int D,
                       int32_t mult, int shift, int zp);
/* s8 A x u8 B HMX-field GEMM (i8_conv2d_1x1_hmx/reference.c,
 * i8_pointwise_conv_hmx/reference.c): store ORACLE_HMX_STORE_I32 (sx12),
 * _U16_FIELD or _ACC_I32. */
void oracle_gemm_hmx_s8u8_rows(const int8_t *A, const uint8_t *B, void *out, int store, int M,
                               int N, int K, int r0, int r1);

/* kernels/expert/requant_per_channel/reference.c:2-17 (rows = channels) */
void oracle_requant_per_channel(const int32_t *a, int8_t *out, int R, int C,
                                const int32_t *mult, const int *shift, int8_t zp);

/* kernels/expert/requantize_i32_u8_dma/reference.c:5-18 */
void oracle_requantize_i32_u8(const int32_t *a, uint8_t *out, int64_t n,
                              int32_t mult, int shift, uint8_t zp);

/* Elementwise requant family (one restatement, parameters per bundle):
 *   x = a                       (pre A)           requantize_i32_i8_dma, epilogue_requant_i32_i8,
 *                                                 requant_relu_dma, requant_relu6_dma,
 *                                                 i8_clip_requant_dma, requant_sigmoid_lut,
 *                                                 requant_tanh_lut, dma_stream_requant_i32_i8
 *   x = a + b                   (pre ADD)         bias_add_requant, residual_add_requant, requant_add_dma
 *   x = max(a + b, 0)           (pre ADD_RELU)    add_relu_requant, i8_skip_add_relu_requant
 *   x = a * b + c               (pre MUL_ADD)     mul_add_requant_dma (c = 50), i8_mul_requant_dma (c = 0)
 *   r = round_half_away(x * mult, shift) + zp   (int64; sign_of_a: sign(a) *
 *       ((|a| * mult + half) >> shift), dma_stream_requant_i32_i8/reference.c)
 *   r = max(min(r, hi1), lo1); r = max(min(r, hi2), lo2)
 *   out = lut ? lut[(uint8)r] : (uint8)r
 * a and b are int32, or int8 when a_i8 / b_kind == 2 (b_kind 0: none,
 * 1: int32).  (kernels/expert/<bundle>/reference.c) */
enum { ORACLE_RQ_PRE_A = 0, ORACLE_RQ_PRE_ADD = 1, ORACLE_RQ_PRE_ADD_RELU = 2,
       ORACLE_RQ_PRE_MUL_ADD = 3 };
void oracle_requant_ew(const void *a, int a_i8, const void *b, int b_kind, int64_t n, int pre,
                       int64_t pre_c, int32_t mult, int shift, int zp, int sign_of_a,
                       int lo1, int hi1, int lo2, int hi2, const int8_t *lut, void *out);
/* epilogue_bias_i32/reference.c: out[r][c] = acc[r][c] + bias[c] (int32, wrap) */
void oracle_epilogue_bias_i32(const int32_t *acc, const int32_t *bias, int32_t *out, int R, int C);
/* epilogue_relu_i8/reference.c: out = max(x, 0) */
void oracle_relu_i8(const int8_t *x, int8_t *out, int64_t n);

/* ---- fp16 GEMM ---- */

/* kernels/expert/fp16_attention_qkt_hmx/reference.c:7-15 generalised to
 * M x N x K: out[i*N+j] = (fp16) sum_d A[i*K+d] * Bt[j*K+d], fp32 accumulate
 * in d order, one fp16 rounding. */
void oracle_gemm_f16_nt_rows(const uint16_t *A, const uint16_t *Bt, uint16_t *out,
                             int M, int N, int K, int r0, int r1);

/* kernels/expert/hmx_matmul_fp16_deepk/reference.c:19-27 generalised to
 * M x N x K with row-major B[K][N]. */
void oracle_gemm_f16_nn_rows(const uint16_t *A, const uint16_t *B, uint16_t *out,
                             int M, int N, int K, int r0, int r1);

/* fp16 GEMM with post-ops, fp32 accumulation in k order starting from
 * res[i][j] (hmx_tile_mac_fp16_32/reference.c) or 0, then + bias[j]
 * (hmx_matmul_fp16_bias), optional rounding to fp16 (preround), the
 * activation act (0 none, 1 relu: hmx_matmul_fp16_relu, 2 leaky x0.125:
 * fp16_matmul_leaky_relu_hmx, 3 tanh gelu: fp16_matmul_gelu_hmx), * scale
 * (qkt_tile_fp16), one final fp16 rounding.  B [K][N], or Bt [N][K] when
 * b_transposed (av_tile_fp16, hmx_conv1x1_fp16). */
void oracle_gemm_f16_ex_rows(const uint16_t *A, const uint16_t *B, int b_transposed,
                             const uint16_t *bias, const uint16_t *res, uint16_t *out, int M,
                             int N, int K, int act, int preround, float scale, int r0, int r1);

/* ---- fp16 attention ---- */

/* kernels/expert/fp16_flash_attention_tile/reference.c:9-28 with the scale
 * as a parameter, heap score buffers (no SK <= 64 cap), an optional causal
 * window (key j visible to query i iff j <= i, top-left aligned) and a loop
 * over BH heads: Q and O are [BH, SQ, D], K and V are [BH, SK, D].
 * Heads [h0, h1) of the flattened B*H range. */
void oracle_attn_f16_heads(const uint16_t *Q, const uint16_t *K,
                           const uint16_t *V, uint16_t *O, int BH, int SQ,
                           int SK, int D, float scale, int causal, int h0,
                           int h1);

/* One head, query rows [q0, q1) only (bounded CPU samples).  Q and O point
 * at the head's row 0; K and V at the head's key 0. */
void oracle_attn_f16_head_rows(const uint16_t *Q, const uint16_t *K,
                               const uint16_t *V, uint16_t *O, int SK, int D,
                               float scale, int causal, int q0, int q1);

/* kernels/expert/online_softmax_step_fp16/kernel_api.h:17-24 recurrence,
 * restated from its reference.c */
void oracle_online_softmax_step_f16(const uint16_t *scores, const uint16_t *V,
                                    uint16_t *running_max, uint16_t *running_sum,
                                    uint16_t *acc, int BLK, int D);

/* ---- row reductions ---- */

/* kernels/expert/fp16_softmax/reference.c:8-29 in fp32 (no C <= 256 cap) */
void oracle_softmax_f32_rows(const float *x, float *out, int R, int C,
                             int r0, int r1);
/* same, fp16 storage, exactly reference.c:8-29 */
void oracle_softmax_f16_rows(const uint16_t *x, uint16_t *out, int R, int C,
                             int r0, int r1);

/* kernels/expert/fp16_layernorm/reference.c:7-24 applied per row of an R x C
 * matrix with eps as a parameter (the reference hardwires 1e-3f). */
void oracle_layernorm_f32_rows(const float *x, const float *gamma,
                               const float *beta, float *out, int R, int C,
                               float eps, int r0, int r1);
void oracle_layernorm_f16_rows(const uint16_t *x, const uint16_t *gamma,
                               const uint16_t *beta, uint16_t *out, int R,
                               int C, float eps, int r0, int r1);

/* kernels/expert/fp16_rmsnorm/reference.c:6-17 per row, eps parameter
 * (the reference hardwires 1e-3f). */
void oracle_rmsnorm_f32_rows(const float *x, const float *gamma, float *out,
                             int R, int C, float eps, int r0, int r1);
void oracle_rmsnorm_f16_rows(const uint16_t *x, const uint16_t *gamma,
                             uint16_t *out, int R, int C, float eps, int r0,
                             int r1);

/* kernels/mined/fp32_sum/reference.c:6-17 (sequential fp32 accumulate) per
 * row; op 0 = sum, op 1 = max (fp32_max_other style max, NaN-free inputs). */
void oracle_rowreduce_f32_rows(const float *x, float *out, int R, int C,
                               int op, int r0, int r1);

/* ---- threaded drivers: split [0, rows) into nthreads contiguous blocks ---- */
/* Whole-array integer reductions, each a plain left-to-right scan as in
 * kernels/expert/<bundle>/reference.c (int32 sums wrap modulo 2^32, the
 * references' signed int32 accumulators on a two's-complement machine):
 * elem ORACLE_ELEM_*, op ORACLE_RED_* (same numbering as hexcuda.h's
 * HEXCUDA_ELEM_* / HEXCUDA_RED_*).  out: int32[1], int64[1] (SUM64) or
 * int32[2] (TOP1). */
enum { ORACLE_ELEM_I8 = 0, ORACLE_ELEM_U8 = 1, ORACLE_ELEM_I16 = 2, ORACLE_ELEM_I32 = 3 };
enum {
    ORACLE_RED_SUM = 0, ORACLE_RED_SUM64, ORACLE_RED_SUMSQ, ORACLE_RED_SUMSQ_DIFF, ORACLE_RED_DOT,
    ORACLE_RED_L1, ORACLE_RED_ABSMAX, ORACLE_RED_MAX, ORACLE_RED_MIN, ORACLE_RED_ARGMAX,
    ORACLE_RED_ARGMIN, ORACLE_RED_TOP1, ORACLE_RED_MEAN
};
void oracle_reduce_int(const void *a, const void *b, int elem, int64_t n, int op, void *out);
/* out[i] = max / min (op 0 / 1) of a[i] and b[i], or of a[i] and c (b null). */
void oracle_minmax_ew(const void *a, const void *b, int32_t c, int elem, int op, void *out,
                      int64_t n);
/* out[k] = sum_{j < w} a[w k + j] (hvx_vradd_i8_reduce/reference.c, w = 4). */
void oracle_group_sum_i8(const int8_t *a, int32_t *out, int64_t g, int w);
/* out[k] = sum_{j < w} a[w k + j] b[w k + j] (hvx_vrmpy_i8_dot/reference.c). */
void oracle_group_dot_i8(const int8_t *a, const int8_t *b, int32_t *out, int64_t g, int w);
/* sat8(round_half_away(lut[gate + 128] up * mult >> shift))
 * (mlp_gate_silu_i8/reference.c). */
void oracle_gate_mul_requant_i8(const int8_t *gate, const int8_t *up, const int8_t *lut,
                                int8_t *out, int64_t n, int32_t mult, int shift);
/* inclusive prefix max from -128 (i8_scan_max/reference.c). */
void oracle_scan_max_i8(const int8_t *in, int8_t *out, int64_t n);
/* gqa_group_reduce_i8/reference.c: sum of a group's H/G head planes, requant. */
void oracle_head_group_reduce_i8(const int8_t *X, int8_t *Y, int H, int G, int64_t MN,
                                 int32_t mult, int shift);

/* int8 layernorm with an inverse-variance table (affine 0 shared gamma[j],
 * 1 rowwise gamma[r W + j], 2 per-row gamma[r] with the table inv_lut + 256 r;
 * idx: gathered rows; res: saturating residual first).
 * kernels/expert/{i8_layernorm_dma,i8_instance_norm,i8_chunk_norm,
 * layernorm_residual,embedding_layer_norm}/reference.c */
void oracle_layernorm_lut_i8(const int8_t *x, const int32_t *idx, const int8_t *res, int8_t *out,
                             int R, int W, const int8_t *gamma, const int8_t *beta,
                             const uint8_t *inv_lut, int affine);
/* layernorm_row_i16/reference.c (order 0), layernorm_affine_i16/reference.c (1) */
void oracle_layernorm_lut_i16(const int16_t *x, int16_t *out, int R, int C, const int16_t *gamma,
                              const int16_t *beta, const uint16_t *inv_lut, int order);
/* row softmax by an exp table: i8_gemm_softmax_tile/reference.c step C (u8),
 * vtcm_softmax_row_i16/reference.c (i16) */
void oracle_lut_softmax_u8(const int8_t *x, uint8_t *out, int R, int C, const uint8_t *exp_lut,
                           const uint16_t *recip_lut);
/* rmsnorm_gain_fp16/reference.c: one gain per row */
void oracle_rmsnorm_gain_f16(const uint16_t *x, const uint16_t *gain, uint16_t *out, int R, int C,
                             float eps);
void oracle_lut_softmax_i16(const int16_t *x, int16_t *out, int R, int C, const uint16_t *exp_lut);
/* attention_scale_i16/reference.c */
void oracle_requant_i16(const int32_t *a, int16_t *out, int64_t n, int32_t mult, int shift);
/* i8_norm_requant_dma/reference.c:11-32 with the channel count and tables as
 * parameters */
void oracle_norm_requant_i8(const int8_t *a, int8_t *out, int64_t n, int nch, const int32_t *nmult,
                            const int *nshift, int32_t mult, int shift, int zp);

enum {
    ORACLE_OP_I8_GEMM_REQUANT = 1,
    ORACLE_OP_GEMM_U8S8_PC = 2,
    ORACLE_OP_GEMM_F16_NT = 3,
    ORACLE_OP_ATTN_F16 = 4,
    ORACLE_OP_SOFTMAX_F32 = 5,
    ORACLE_OP_LAYERNORM_F32 = 6,
    ORACLE_OP_ROWREDUCE_F32 = 7,
};
/* Runs `op` with its arguments packed in `args` (see hexoracle.c) over rows
 * (or heads) [r0, r1) split across nthreads pthreads.  Returns 0 on success. */
int oracle_parallel(int op, const void *args, int r0, int r1, int nthreads);

/* Packed argument blocks for oracle_parallel */
typedef struct {
    const void *A, *B; const int32_t *bias; void *out;
    int M, N, K; int32_t zpA; int32_t mult; int shift; int zp;
    const int32_t *mult_pc; const int *shift_pc;
} oracle_gemm_args;
typedef struct {
    const uint16_t *Q, *K, *V; uint16_t *O; int BH, SQ, SK, D; float scale; int causal;
} oracle_attn_args;
typedef struct {
    const float *x, *gamma, *beta; float *out; int R, C; float eps; int op;
} oracle_rows_args;

/* kernels/expert/kv_cache_update/reference.c: row pos of each head's caches. */
void oracle_kv_cache_update_i8(int8_t *k_cache, int8_t *v_cache, const int8_t *k_new,
                               const int8_t *v_new, int pos, int heads, int cache_len,
                               int head_dim);
/* kernels/expert/rope_pair_fp16/reference.c: interleaved-pair rotation. */
void oracle_rope_pair_f16(const uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                          uint16_t *out, int64_t n_pairs);

/* kernels/expert/i8_ffn_block/reference.c: HMX-field FFN, ReLU + shift. */
void oracle_ffn_hmx_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2,
                       const int32_t *b2, int8_t *out, int M, int D, int Dff, int sh1, int sh2);
/* kernels/expert/i8_ffn_swiglu_block/reference.c: HMX-field SwiGLU FFN. */
void oracle_ffn_swiglu_hmx_i8(const uint8_t *X, const int8_t *Wg, const int8_t *Wu,
                              const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut,
                              int8_t *out, int M, int D, int Dff, int sg, int su, int sh, int zp,
                              int so);
/* kernels/expert/i8_transformer_encoder_block/reference.c. */
void oracle_encoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut,
                             int8_t *out, int S, int D, int Dff);

/* clamp(round((x - zp_in) * mult + add, shift) + zp_out, lo, hi); round 0
 * half away from zero, 1 floor; wrap32: int32 product and sum (the
 * rescale / dequant / HMX-store / bias-add / affine bundles' reference.c). */
void oracle_affine_ew(const void *in, int elem_in, void *out, int elem_out, int64_t n, int32_t zp_in,
                      int32_t mult, int64_t add, int shift, int round, int wrap32, int zp_out,
                      int32_t lo, int32_t hi);

/* kernels/expert/i16_gemm/reference.c: int16 GEMM, int32 accumulator. */
void oracle_gemm_i16(const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K);

/* kernels/expert/i8_channel_mix_block/reference.c (lut NULL: no table). */
void oracle_mix_mlp_i8(const int8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *lut,
                       const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V, int D,
                       int32_t mult1, int shift1, int32_t mult2, int shift2);
/* kernels/expert/i8_token_mix_block/reference.c. */
void oracle_token_mix_i8(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2,
                         const int32_t *b2, int8_t *out, int T, int C, int DM, int32_t mult1,
                         int shift1, int32_t mult2, int shift2);
/* kernels/expert/rnn_cell_i8/reference.c. */
void oracle_rnn_cell_i8(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x,
                        const int8_t *h_prev, int8_t *h_t, int H, int I, int32_t mult, int shift,
                        int zp, const int8_t *tanh_lut);

/* HMX-convention convolution (the i8_conv2d_*_hmx / i8_conv1d_bias_requant_hmx
 * reference.c files), no padding. */
void oracle_conv2d_hmx(const uint8_t *in, const int8_t *W, const int32_t *bias, void *out, int store,
                       int act, int c_in, int ih, int iw, int c_out, int kh, int kw, int stride);

#ifdef __cplusplus
}
#endif
#endif /* HEXORACLE_H */
