/* hexcuda.h -- C ABI of libhexcuda, the B200 (sm_100a) implementation of the
 * hexkernels DL-operator hot path.
 *
 * The corpus's drop-in boundary is one C function per task,
 *     void candidate_kernel(...);
 * declared in each bundle's kernel_api.h and called by that bundle's harness.c
 * (sriharshapy/hexkernels: README.md:94-95, e.g.
 * kernels/expert/i8_gemm_requant/kernel_api.h:9-11 and harness.c:55).  The
 * corpus has no other FFI: its Python tooling (hexkernels/core/evaluate.py:
 * 554-567) compiles harness.c + the candidate into one program and parses the
 * HVXENV_* lines it prints.  libhexcuda therefore exports
 *
 *   1. runtime calls (device set, allocation, copies, streams, errors, timing)
 *      that the thin candidate_kernel shims in hexkernels_b200/shims/ use;
 *   2. one DEVICE-POINTER launcher per operator (asynchronous on the device's
 *      stream; inputs and outputs already in HBM);
 *   3. one HOST-POINTER entry per operator (hexcuda_host_*): shards rows over
 *      the initialised devices, copies in, launches, copies out, synchronises.
 *      Each candidate_kernel shim is a one-line call of one of these.
 *
 * Conventions: plain pointers and sizes only; fp16 data is passed as uint16_t
 * bit patterns (IEEE binary16, same bits as the corpus's __fp16); row-major
 * unless stated.  Every entry returns 0 (HEXCUDA_OK) or an error code; on
 * error the host entries leave the caller's output buffer untouched, print one
 * "HEXCUDA_ERROR <code> <message>" line to stderr and record the code for
 * hexcuda_last_error().  Nothing aborts or traps.  Not thread-safe: one caller
 * thread at a time, like the corpus harnesses.
 */
#ifndef HEXCUDA_H
#define HEXCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HEXCUDA_OK 0
#define HEXCUDA_ERR_ARG 1         /* bad size, null pointer, unsupported shape */
#define HEXCUDA_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define HEXCUDA_ERR_NODEV 3       /* no usable sm_100 device / not initialised */
#define HEXCUDA_ERR_TIMEOUT 4     /* a device-side bounded wait expired */
#define HEXCUDA_ERR_OOM 5         /* device or pinned allocation failed */

/* ------------------------------------------------------------------ runtime */

/* Initialise on devices 0..ngpus-1 (ngpus <= 0: all visible devices).
 * Idempotent; a second call with a different set re-initialises. */
int hexcuda_init(int ngpus);
/* Initialise on an explicit device list (e.g. one LOCAL_RANK per process). */
int hexcuda_init_devices(const int *devs, int n);
void hexcuda_shutdown(void);
/* Number of initialised devices; the host entries shard rows over them. */
int hexcuda_device_count(void);
/* CUDA ordinal of initialised device slot `slot`. */
int hexcuda_device_ordinal(int slot);

/* All `dev` arguments below are slots 0..hexcuda_device_count()-1. */
void *hexcuda_alloc(int dev, size_t bytes);
int hexcuda_free(int dev, void *ptr);
void *hexcuda_host_alloc(size_t bytes);       /* pinned host memory */
int hexcuda_host_free(void *ptr);
int hexcuda_h2d(int dev, void *dst, const void *src, size_t bytes);   /* async */
int hexcuda_d2h(int dev, void *dst, const void *src, size_t bytes);   /* async */
int hexcuda_memset(int dev, void *dst, int value, size_t bytes);       /* async */
/* Waits for the device's stream, then checks the device watchdog word.
 * dev < 0: every initialised device. */
int hexcuda_sync(int dev);
/* The device's launch stream (a cudaStream_t).  hexcuda_set_stream installs a
 * caller's stream, e.g. the one a framework is using, as given (NULL is CUDA's
 * legacy default stream); hexcuda_reset_stream returns to libhexcuda's own
 * non-blocking stream. */
void *hexcuda_stream(int dev);
int hexcuda_set_stream(int dev, void *stream);
int hexcuda_reset_stream(int dev);

int hexcuda_last_error(void);
const char *hexcuda_last_error_string(void);
/* Record a cudaEvent pair around each launch (default on).  The device time
 * of the most recent launch (max over devices for a sharded host entry),
 * in ms, or -1 when timing is off or nothing was launched. */
int hexcuda_set_timing(int on);
float hexcuda_last_kernel_ms(void);
/* Number of kernels libhexcuda has launched since load (all devices). */
uint64_t hexcuda_launch_count(void);
/* Kinds of kernel launched since the last reset (reset != 0 clears after
 * reading): bit 0 tcgen05 tensor-core MMA kernels, bit 1 TMA-fed kernels,
 * bit 2 HBM-bound kernels on their 128-bit vector load / store path.
 * The evaluator's mechanism verdict (hexkernels_b200/evaluate.py) reads it
 * around each candidate_kernel call: the B200 counterpart of the reference's
 * used_hvx / used_hmx / used_dma flags (hexkernels/core/evaluate.py:573-597). */
#define HEXCUDA_MECH_TCGEN05 1u
#define HEXCUDA_MECH_TMA 2u
#define HEXCUDA_MECH_VEC128 4u
unsigned hexcuda_mechanisms(int reset);

/* ------------------------------------------ multi-GPU: shards and replicas */

/* The row split every host entry uses over n devices (and bench.py over n
 * ranks): part `part` owns rows [rows*part/n, rows*(part+1)/n).  Pure host
 * arithmetic; needs no device.  The reference has no multi-device code: this
 * and the calls below are the "ngpus / replicate" knob of the drop-in
 * boundary (one C entry per task, kernels/expert/<task>/kernel_api.h). */
int hexcuda_shard_rows(int64_t rows, int nparts, int part, int64_t *r0, int64_t *r1);

/* Replicated outputs.  With replicate on, a host entry over N > 1 devices
 * whose output is row-major also all-gathers the devices' output rows over
 * NVLink (NCCL, opened with dlopen on first use), so that every device holds
 * the whole output in its own memory; hexcuda_replica returns device slot
 * `dev`'s copy (valid until the next host entry).  The host output is still
 * copied from each device's own rows.  Equal parts move in one ncclAllGather,
 * ragged parts in one ncclBroadcast per owning part inside one NCCL group.
 * hexcuda_last_collective_ms: device time of the last gather (max over
 * devices), timed apart from hexcuda_last_kernel_ms.  Off by default. */
int hexcuda_set_replicate(int on);
int hexcuda_get_replicate(void);
int hexcuda_replica(int dev, void **ptr, size_t *bytes);
float hexcuda_last_collective_ms(void);
/* Device-pointer gather, one process over every initialised device: slot i
 * holds rows [rows*i/n, rows*(i+1)/n) at shards[i] (may be null when that part
 * is empty); afterwards fulls[i] (rows * row_bytes on slot i) holds all rows.
 * shards[i] may point into fulls[i] at its own offset (in place).
 * Asynchronous on each device's stream. */
int hexcuda_allgather_rows(const void *const *shards, void *const *fulls, int64_t rows,
                           size_t row_bytes);
/* The same across processes, one GPU per process (one initialised device):
 * rank 0 makes an id (>= 128 bytes), every rank joins with it, then each
 * rank passes its own part and receives all rows. */
int hexcuda_comm_unique_id(void *id, size_t id_bytes);
int hexcuda_comm_init_rank(int nranks, int rank, const void *id, size_t id_bytes);
int hexcuda_comm_destroy(void);
int hexcuda_comm_allgather_rows(const void *shard, void *full, int64_t rows, size_t row_bytes);

/* --------------------------------------------- device-pointer launchers */

/* Row softmax over the last axis of an R x C matrix.
 * kernels/expert/fp16_softmax/kernel_api.h:4-15 (fp32 and fp16 storage). */
int hexcuda_softmax_f32(int dev, const float *x, float *out, int R, int C);
int hexcuda_softmax_f16(int dev, const uint16_t *x, uint16_t *out, int R, int C);

/* Per-row layernorm, mean/var by E[x^2] - mean^2 clamped at 0.
 * kernels/expert/fp16_layernorm/kernel_api.h:4-18 with eps a parameter. */
int hexcuda_layernorm_f32(int dev, const float *x, const float *gamma,
                          const float *beta, float *out, int R, int C, float eps);
int hexcuda_layernorm_f16(int dev, const uint16_t *x, const uint16_t *gamma,
                          const uint16_t *beta, uint16_t *out, int R, int C,
                          float eps);

/* Per-row RMS norm.  kernels/expert/fp16_rmsnorm/reference.c:6-17 with eps a
 * parameter. */
int hexcuda_rmsnorm_f32(int dev, const float *x, const float *gamma, float *out,
                        int R, int C, float eps);
int hexcuda_rmsnorm_f16(int dev, const uint16_t *x, const uint16_t *gamma,
                        uint16_t *out, int R, int C, float eps);
/* Same with one gain per row instead of per-column gamma:
 * kernels/expert/rmsnorm_gain_fp16/reference.c (eps 1e-3 there). */
int hexcuda_rmsnorm_gain_f16(int dev, const uint16_t *x, const uint16_t *gain, uint16_t *out,
                             int R, int C, float eps);

/* Row sum (op 0) or row max (op 1): out[R].  kernels/mined/fp32_sum/
 * reference.c:6-17 per row. */
int hexcuda_rowreduce_f32(int dev, const float *x, float *out, int R, int C, int op);

/* int32 -> int8 per-channel (row) requant.
 * kernels/expert/requant_per_channel/kernel_api.h:4-11. */
int hexcuda_requant_per_channel(int dev, const int32_t *a, int8_t *out, int R,
                                int C, const int32_t *mult, const int *shift,
                                int8_t zp);
/* int32 -> uint8 requant.  kernels/expert/requantize_i32_u8_dma/kernel_api.h:4-14. */
int hexcuda_requantize_i32_u8(int dev, const int32_t *a, uint8_t *out, int64_t n,
                              int32_t mult, int shift, uint8_t zp);

/* Elementwise requant family, n elements:
 *   x = a (pre A) | a + b (ADD) | max(a + b, 0) (ADD_RELU) | a * b + pre_c (MUL_ADD)
 *   r = round_half_away((int64) x * mult >> shift) + zp       (shift 0..63)
 *       with sign_of_a: sign(x) * ((|x| * mult + half) >> shift)
 *   r = max(min(r, hi1), lo1); r = max(min(r, hi2), lo2)
 *   out byte = lut ? lut[(uint8) r] : (uint8) r
 * a int32 (or int8 with a_i8), b none / int32 / int8 (b_kind 0 / 1 / 2).
 * zp, lo1, hi1, lo2, hi2 within +-2^24; the two-operand forms take a and b
 * both int32 or both int8; sign_of_a only with pre A (HEXCUDA_ERR_ARG otherwise).
 * Products that leave int64 wrap (undefined in the C references).
 * Bundles (kernels/expert/<name>/kernel_api.h): requantize_i32_i8_dma,
 * epilogue_requant_i32_i8, requant_relu_dma (13, 3, clamp [0,127]),
 * requant_relu6_dma (clamp [0,24]), i8_clip_requant_dma (second clamp
 * [lo,hi]), dma_stream_requant_i32_i8 (sign_of_a), requant_sigmoid_lut and
 * requant_tanh_lut (clamp [0,255], table), bias_add_requant,
 * residual_add_requant, requant_add_dma (5, 3), add_relu_requant,
 * i8_skip_add_relu_requant, mul_add_requant_dma (pre_c 50, 3, 1),
 * i8_mul_requant_dma. */
#define HEXCUDA_RQ_PRE_A 0
#define HEXCUDA_RQ_PRE_ADD 1
#define HEXCUDA_RQ_PRE_ADD_RELU 2
#define HEXCUDA_RQ_PRE_MUL_ADD 3
int hexcuda_requant_ew(int dev, const void *a, int a_i8, const void *b, int b_kind,
                       void *out, int64_t n, int pre, int64_t pre_c, int32_t mult,
                       int shift, int zp, int sign_of_a, int lo1, int hi1, int lo2,
                       int hi2, const int8_t *lut);
/* out[r][c] = acc[r][c] + bias[c], int32 (wrap).
 * kernels/expert/epilogue_bias_i32/kernel_api.h:14. */
int hexcuda_epilogue_bias_i32(int dev, const int32_t *acc, const int32_t *bias,
                              int32_t *out, int R, int C);
/* out = max(x, 0), int8.  kernels/expert/epilogue_relu_i8/kernel_api.h:13. */
int hexcuda_relu_i8(int dev, const int8_t *x, int8_t *out, int64_t n);

/* Whole-array integer reductions over n elements of a (and b), one scalar
 * result.  elem: HEXCUDA_ELEM_I8 / _U8 / _I16 / _I32.  Sums wrap modulo 2^32
 * like the references' int32 accumulators, SUM64 accumulates in int64:
 *   SUM       out i32 = sum a[i]             vtcm_reduce_i32 (i32), i8_sum_dma
 *   SUM64     out i64 = sum a[i]             dma_double_buffer_reduce_i32
 *   SUMSQ     out i32 = sum a[i]^2           i8_sumsq_i32
 *   SUMSQ_DIFF out i32 = sum (a[i]-b[i])^2   i8_sumsq_diff_i32
 *   DOT       out i32 = sum a[i]*b[i]        i8_weighted_sum
 *   L1        out i32 = sum |a[i]|           i8_l1norm_dma
 *   ABSMAX    out i32 = max(0, max |a[i]|)   i8_absmax_dma
 *   MAX / MIN out i32 = max / min a[i]       dma_stream_max_u8 (u8, 0 when n = 0)
 *   ARGMAX / ARGMIN out i32 = first index of the max / min   i8_argmax_dma, i8_argmin_dma
 *   TOP1      out i32[2] = {max, first index of it}          i8_top1_reduce_dma
 *   MEAN      out i32 = (int32 sum) / n, truncated (C /)     i8_mean_dma
 * (kernels/expert/<bundle>/reference.c).  ARGMAX, ARGMIN, TOP1 and MEAN need
 * n >= 1 (the references read a[0] / divide by n).  out is a device pointer. */
#define HEXCUDA_ELEM_I8 0
#define HEXCUDA_ELEM_U8 1
#define HEXCUDA_ELEM_I16 2
#define HEXCUDA_ELEM_I32 3
#define HEXCUDA_RED_SUM 0
#define HEXCUDA_RED_SUM64 1
#define HEXCUDA_RED_SUMSQ 2
#define HEXCUDA_RED_SUMSQ_DIFF 3
#define HEXCUDA_RED_DOT 4
#define HEXCUDA_RED_L1 5
#define HEXCUDA_RED_ABSMAX 6
#define HEXCUDA_RED_MAX 7
#define HEXCUDA_RED_MIN 8
#define HEXCUDA_RED_ARGMAX 9
#define HEXCUDA_RED_ARGMIN 10
#define HEXCUDA_RED_TOP1 11
#define HEXCUDA_RED_MEAN 12
int hexcuda_reduce_int(int dev, const void *a, const void *b, int elem, int64_t n, int op,
                       void *out);

/* int8 layernorm with an inverse-variance table, one row of W elements per
 * output row r < R:  t = x row (row idx[r] of x when idx is not NULL; t =
 * sat8(t + res[r][j]) when res is not NULL); mu = sum t / W; var = sum (t -
 * mu)^2 / W (int32, C division); inv = lut[clamp(var, 0, 255)];
 * out = sat8(((((t - mu) g + 64) >> 7) inv + 128) >> 8) + b).
 * affine SHARED: g = gamma[j], b = beta[j] (i8_layernorm_dma, layernorm_residual,
 * embedding_layer_norm); ROWWISE: gamma[r W + j] (i8_chunk_norm); PER_ROW:
 * gamma[r], beta[r] and the table inv_lut + 256 r (i8_instance_norm). */
#define HEXCUDA_LN_AFFINE_SHARED 0
#define HEXCUDA_LN_AFFINE_ROWWISE 1
#define HEXCUDA_LN_AFFINE_PER_ROW 2
/* RMS form (rmsnorm_residual): mu = 0, var = sum t^2 / W, out =
 * sat8((((t g[j] + 64) >> 7) inv + 128) >> 8); beta unused (may be NULL). */
#define HEXCUDA_LN_RMS_SHARED 3
int hexcuda_layernorm_lut_i8(int dev, const int8_t *x, const int32_t *idx, const int8_t *res,
                             int8_t *out, int R, int W, const int8_t *gamma, const int8_t *beta,
                             const uint8_t *inv_lut, int affine);
/* int16 forms: mu = (int32)(sum / C), var = sum (x - mu)^2 / C (int64),
 * inv = inv_lut[clamp(var >> 5, 0, 255)]; order 0 (layernorm_row_i16):
 * sat16(((((x - mu) gamma[c] + 32) >> 6) inv + 512) >> 10) + beta[c]);
 * order 1 (layernorm_affine_i16): sat16(((((x - mu) inv + 512) >> 10)
 * gamma[r] + 32) >> 6) + beta[r]). */
int hexcuda_layernorm_lut_i16(int dev, const int16_t *x, int16_t *out, int R, int C,
                              const int16_t *gamma, const int16_t *beta, const uint16_t *inv_lut,
                              int order);
/* Row softmax by an exp table: m = row max, e = lut[max(x - m, -255) + 255],
 * S = sum e, p = (e 255 + S / 2) / S as uint8 (i8_gemm_softmax_tile,
 * matmul_softmax_tile step B); the int16 form with a uint16 table, int64 S
 * and (e 32767 + S / 2) / S (vtcm_softmax_row_i16). */
/* recip_lut not NULL (softmax_row_i8): p = clamp((e recip_lut[clamp(S >> 6,
 * 0, 255)] + 32768) >> 16, 0, 255) instead of the division.  softmax_rowwise
 * is the division form. */
int hexcuda_lut_softmax_u8(int dev, const int8_t *x, uint8_t *out, int R, int C,
                           const uint8_t *exp_lut, const uint16_t *recip_lut);
int hexcuda_lut_softmax_i16(int dev, const int16_t *x, int16_t *out, int R, int C,
                            const uint16_t *exp_lut);
/* out = sat16(round_half_away(a * mult >> shift)): attention_scale_i16. */
int hexcuda_requant_i16(int dev, const int32_t *a, int16_t *out, int64_t n, int32_t mult,
                        int shift);
/* Channel c = i / (n / nch) of the first nch (n / nch) elements:
 * v = round_half_away(a * nmult[c] >> nshift[c]) (int64, unclamped),
 * out = sat8(round_half_away(v * mult >> shift) + zp): i8_norm_requant_dma
 * (16 channels, its fixed tables, 5 / 4 / 0). */
int hexcuda_norm_requant_i8(int dev, const int8_t *a, int8_t *out, int64_t n, int nch,
                            const int32_t *nmult, const int *nshift, int32_t mult, int shift,
                            int zp);
/* s8 GEMM -> int8 scores (sat8 of the accumulator, or with requant the
 * round-half-away requant by mult / shift) -> hexcuda_lut_softmax_u8:
 * i8_gemm_softmax_tile (B row-major), matmul_softmax_tile (K as Bt, requant). */
int hexcuda_gemm_softmax_u8(int dev, const int8_t *A, const int8_t *B, int b_transposed,
                            const uint8_t *exp_lut, uint8_t *out, int M, int N, int K,
                            int requant, int32_t mult, int shift);
/* gelu_ffn_residual: hid = gelu_lut[sat8(x W1 + b1) + 128]; s = sat8(hid W2 +
 * b2 + x_res); out = hexcuda_layernorm_lut_i8(s, gamma, beta, inv_lut)
 * (W1 [K,V], W2 [V,D] row-major; the intermediates stay in HBM). */
int hexcuda_gelu_ffn_residual_i8(int dev, const int8_t *x, const int8_t *W1, const int32_t *b1,
                                 const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2,
                                 const int8_t *x_res, const int8_t *gamma, const int8_t *beta,
                                 const uint8_t *inv_lut, int8_t *out, int M, int K, int V, int D);

/* Elementwise max (op 0) or min (op 1) of a[i] and b[i], or of a[i] and the
 * scalar c when b is null: hvx_vmax_i8, hvx_vmax_u8, hvx_vmin_i16,
 * hvx_vmin_u8, i8_max_scalar_dma, i8_min_scalar_dma.  elem I8, U8 or I16. */
int hexcuda_minmax_ew(int dev, const void *a, const void *b, int32_t c, int elem, int op,
                      void *out, int64_t n);

/* out[k] = sum_{j < w} a[w k + j] for k < g (int8 -> int32), w >= 1:
 * hvx_vradd_i8_reduce (w = 4). */
int hexcuda_group_sum_i8(int dev, const int8_t *a, int32_t *out, int64_t g, int w);
/* out[k] = sum_{j < w} a[w k + j] b[w k + j] (int32, modulo 2^32):
 * kernels/expert/hvx_vrmpy_i8_dot/reference.c:3-9 (w = 4). */
int hexcuda_group_dot_i8(int dev, const int8_t *a, const int8_t *b, int32_t *out, int64_t g, int w);
/* out = sat8(round_half_away((lut[gate + 128] up) * mult >> shift)), n
 * elements: the SiLU-gated product of kernels/expert/mlp_gate_silu_i8/
 * reference.c:4-15. */
int hexcuda_gate_mul_requant_i8(int dev, const int8_t *gate, const int8_t *up, const int8_t *lut,
                                int8_t *out, int64_t n, int32_t mult, int shift);

/* Inclusive prefix maximum, out[i] = max(-128, in[0..i]): i8_scan_max. */
int hexcuda_scan_max_i8(int dev, const int8_t *in, int8_t *out, int64_t n);

/* Head-group reduce: Y[g][i] = sat_i8(round_half_away(sum_{t < heads/G}
 * X[g heads/G + t][i] * mult >> shift)) for g < G, i < MN: gqa_group_reduce_i8
 * (reference.c: sum of the group's head planes, requant, clamp). */
int hexcuda_head_group_reduce_i8(int dev, const int8_t *X, int8_t *Y, int heads, int G,
                                 int64_t MN, int32_t mult, int shift);

/* int8 GEMM + requant: A [M,K] s8, B [K,N] s8 row-major, out [M,N] s8.
 * kernels/expert/i8_gemm_requant/kernel_api.h:4-11. */
int hexcuda_gemm_i8_requant(int dev, const int8_t *A, const int8_t *B, int8_t *out,
                            int M, int N, int K, int32_t mult, int shift, int8_t zp);
/* + per-column int32 bias before the requant.
 * kernels/expert/i8_gemm_bias_requant/kernel_api.h:4-18. */
int hexcuda_gemm_i8_bias_requant(int dev, const int8_t *A, const int8_t *B,
                                 const int32_t *bias, int8_t *out, int M, int N,
                                 int K, int32_t mult, int shift, int8_t zp);
/* zero-point decomposition acc = A.B - zpA * colsum(B), no output zp.
 * kernels/expert/gemm_tile_zp_i8/kernel_api.h:4-28. */
int hexcuda_gemm_i8_zp(int dev, const int8_t *A, const int8_t *B, int8_t *out,
                       int M, int N, int K, int32_t zpA, int32_t scale_mult,
                       int scale_shift);
/* u8 x s8 asymmetric GEMM, per-output-channel requant to u8:
 * acc = A.B - zpA * colsum(B); biased = acc + bias[j];
 * out = sat_u8(round_half_away(biased * mult[j] >> shift[j]) + zp_out).
 * Composition of gemm_tile_zp_i8/reference.c:10-19, i8_gemm_bias_requant/
 * reference.c:13, requant_per_channel/reference.c:5-10 and
 * requantize_i32_u8_dma/reference.c:5-13; candidate_kernel header
 * include/kernel_api/gemm_u8s8_pc.h. */
int hexcuda_gemm_u8s8_pc(int dev, const uint8_t *A, const int8_t *B,
                         const int32_t *bias, uint8_t *out, int M, int N, int K,
                         int32_t zpA, const int32_t *mult, const int *shift,
                         uint8_t zp_out);

/* Same operator, for callers that cannot have the library allocate device
 * memory (a runtime that reserved the GPU's memory for its own arena, where a
 * library cudaMalloc would fail; a latency-bound caller that cannot take
 * cudaMalloc's implicit synchronisation).  This entry has no counterpart in
 * the reference; it calls no cudaMalloc / cudaFree.  Its scratch (a K-major
 * copy of B and the column sums) is a fixed region compiled into libhexcuda
 * that every GPU loading the library holds until exit: limits
 * round_up(K, 128) * N <= 16 MiB and N <= 16384; A rows must be 16-byte
 * aligned (K % 16 == 0, K >= 128).  Other shapes return HEXCUDA_ERR_ARG.
 * The first call on a device looks up the region's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  All calls share the region and it keeps the
 * last call's contents (the column sums are cleared on every call): calls
 * that overlap on the GPU, from different streams, race on it. */
int hexcuda_gemm_u8s8_pc_noalloc(int dev, const uint8_t *A, const int8_t *B,
                                 const int32_t *bias, uint8_t *out, int M, int N,
                                 int K, int32_t zpA, const int32_t *mult,
                                 const int *shift, uint8_t zp_out);

/* HMX-convention u8 x s8 GEMM.  acc = sum_k (A[i][k] - zpA) * B[k][j] in
 * int32 (two's-complement wrap), r = sx12((acc * 17 + 8) >> 4) -- the low 12
 * bits of the matrix engine's 0x40-config requant field, sign-extended -- and
 * by out_kind:
 *   HEXCUDA_HMX_OUT_I32           out int32 [M,N] = r
 *       (kernels/.../hmx_matmul_i8_64/kernel_api.h, hmx_matmul_i8_deepk,
 *        hmx_matmul_i8_zp, hmx_matmul_i8_transposeB)
 *   HEXCUDA_HMX_OUT_I8            out int8 = clamp(r, -128, 127)
 *       (hmx_matmul_i8_requant/kernel_api.h)
 *   HEXCUDA_HMX_OUT_U8_BIAS_RELU  out uint8 = clamp(max(r + bias[j], 0), 0, 255),
 *       r + bias[j] in int32 with wrap (i8_gemm_bias_relu_requant_hmx/kernel_api.h)
 * A uint8 [M,K] row-major.  B int8 [K,N] row-major, or with b_transposed
 * Bt [N,K] (B column-major).  bias is read only for HEXCUDA_HMX_OUT_U8_BIAS_RELU. */
#define HEXCUDA_HMX_OUT_I32 0
#define HEXCUDA_HMX_OUT_I8 1
#define HEXCUDA_HMX_OUT_U8_BIAS_RELU 2
int hexcuda_gemm_hmx(int dev, const uint8_t *A, const int8_t *B, int b_transposed,
                     const int32_t *bias, void *out, int out_kind, int M, int N, int K,
                     int32_t zpA);

/* The HMX-convention GEMM with the post-ops of the rest of that family:
 * v = sx12((acc * 17 + 8) >> 4); v += bias[j] (bias may be NULL);
 * v += res[i][j] (res_kind INT32 or INT8, row-major [M,N]); activation;
 * then the store.  Adds wrap in int32 as the reference's int arithmetic.
 *   store I32           out int32 = v
 *         I8_SAT        out int8 = clamp(v, -128, 127)
 *         U8_SAT        out uint8 = clamp(v, 0, 255)
 *         I8_LOW        out int8 = low 8 bits of v (i8_matmul_hmx_requant)
 *         U16_FIELD     out uint16 = v & 0xFFF, the unsigned 12-bit field
 *                       (hvx_hmx_requant_0x40, env/harness/harness_common.h:127;
 *                       i8_matmul_hmx_64x64, i8_matmul_hmx_96x96)
 *         LUT_I32       out int32 = lut[clamp(v + 128, 0, 255)] (256 int32;
 *                       hmx_matmul_i8_gelu_lut, whose reference is undefined
 *                       outside the table)
 *         LUT_I8        out int8 = lut[clamp(v, -128, 127) + 128] (256 int8;
 *                       i8_matmul_bias_gelu_hmx)
 *   act   RELU max(v, 0); LEAKY_SHR3 v >= 0 ? v : v >> 3 (i8_matmul_leaky_relu_hmx)
 *   col_major  out[j * M + i] (hmx_matmul_i8_col_major)
 * Bundles (kernels/expert/<name>/kernel_api.h): hmx_matmul_i8_{32, accum_chain,
 * bias, bias_relu, col_major, gelu_lut, multi_n, rect_32x64, relu},
 * i8_matmul_{bias, bias_relu, leaky_relu, residual, add_requant, bias_gelu}_hmx,
 * i8_matmul_hmx_{64x64, 96x96, requant}, i8_gemm_relu_hmx_deepk,
 * i8_linear_proj_hmx (W = Bt, b_transposed), hmx_kacc_i8_{2tile, 4tile},
 * hmx_tile_mac_i8_32, hmx_gemv_i8 (N = 1). */
#define HEXCUDA_HMX_STORE_I32 0
#define HEXCUDA_HMX_STORE_I8_SAT 1
#define HEXCUDA_HMX_STORE_U8_SAT 2
#define HEXCUDA_HMX_STORE_I8_LOW 3
#define HEXCUDA_HMX_STORE_U16_FIELD 4
#define HEXCUDA_HMX_STORE_LUT_I32 5
#define HEXCUDA_HMX_STORE_LUT_I8 6
/* out int32 = the accumulator itself, without the 12-bit field (a building
 * block for compositions such as hexcuda_attn_qkt_av_hmx) */
#define HEXCUDA_HMX_STORE_ACC_I32 7
#define HEXCUDA_HMX_ACT_NONE 0
#define HEXCUDA_HMX_ACT_RELU 1
#define HEXCUDA_HMX_ACT_LEAKY_SHR3 2
#define HEXCUDA_HMX_RES_NONE 0
#define HEXCUDA_HMX_RES_I32 1
#define HEXCUDA_HMX_RES_I8 2
int hexcuda_gemm_hmx_ex(int dev, const uint8_t *A, const int8_t *B, int b_transposed,
                        const int32_t *bias, const void *res, int res_kind,
                        const void *lut, void *out, int store, int act, int col_major,
                        int M, int N, int K, int32_t zpA);

/* HMX-convention QK^T -> AV block: Sc = sx12((Q K^T * 17 + 8) >> 4) (int,
 * Q [SQ,D] u8, K [SK,D] s8), out [SQ,D] int32 = sx12((Sc V * 17 + 8) >> 4)
 * (V [SK,D] s8).  kernels/expert/i8_attention_qkt_av_hmx/kernel_api.h
 * (SQ = SK = S).  Four tcgen05 GEMM launches and two elementwise passes; the
 * 12-bit Sc is split exactly into a u8 low byte and a zero-pointed u8 high
 * byte for the second product. */
int hexcuda_attn_qkt_av_hmx(int dev, const uint8_t *Q, const int8_t *K, const int8_t *V,
                            int32_t *out, int SQ, int SK, int D);

/* int8 attention with the corpus's LUT softmax (per score row: m = max;
 * e_j = exp_lut[max(s_j - m, -255) + 255]; p_j = (e_j * 255 + S / 2) / S,
 * S = sum e_j; a row whose S is 0 gets p = 0).  Q [HQ][S][D], K / V
 * [HKV][S][D], query head h uses KV head h / (HQ / HKV); out [HQ][S][D].
 *   REQUANT   Q int8; s = requant_i8(Q.K, scale_mult, scale_shift); out int8 =
 *             requant_i8(P.V, av_mult, av_shift) (round half away, no zero
 *             point).  kernels/expert/gqa_attention/kernel_api.h:40-46.
 *   HMX       Q u8; s = clamp_i8(sx12(HMX field of Q.K) >> 4); out uint16 = HMX
 *             field of P.V.  i8_attention_block/kernel_api.h:30,
 *             i8_gqa_attention_block/kernel_api.h:40.
 *   HMX_ROPE  HMX after rotating each (d, d + D/2) pair of Q and K by the
 *             row's int8 cos / sin tables ([S][D/2]) with >> rot_shift
 *             (clamped to u8 / int8).  i8_rope_attention_block/kernel_api.h:40.
 * One CTA per query head, all operands in shared memory (HEXCUDA_ERR_ARG when
 * S and D need more than 200 KB). */
#define HEXCUDA_ATTN_LUT_REQUANT 0
#define HEXCUDA_ATTN_LUT_HMX 1
#define HEXCUDA_ATTN_LUT_HMX_ROPE 2
int hexcuda_attn_lut_i8(int dev, int mode, const void *Q, const int8_t *K, const int8_t *V,
                        const uint8_t *exp_lut, const int8_t *cos_lut, const int8_t *sin_lut,
                        int rot_shift, void *out, int HQ, int HKV, int S, int D,
                        int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift);
/* The REQUANT form (H query heads, one KV head each) with a banded mask:
 * scores of keys with |i - j| > window are set to -128 and stay in the
 * softmax.  kernels/expert/i8_sparse_attn_block/reference.c:33-42. */
int hexcuda_attn_lut_i8_window(int dev, const int8_t *Q, const int8_t *K, const int8_t *V,
                               const uint8_t *exp_lut, int8_t *out, int heads, int S, int D, int window,
                               int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift);
/* Integer affine elementwise requant: out[i] = clamp(round((x[i] - zp_in) *
 * mult + add, shift) + zp_out, lo, hi), x and out of the HEXCUDA_ELEM_*
 * types; round HEXCUDA_ROUND_HALF_AWAY (sign-magnitude, half away from zero)
 * or HEXCUDA_ROUND_FLOOR (arithmetic right shift); wrap32 != 0 takes the
 * product and sum modulo 2^32 first (the references' int32 arithmetic;
 * shift 0..31), else exactly in int64 (shift 0..62).  kernels/expert/
 * rescale_i16_i8_dma, dequant_i8_i16_dma, hmx_requant_store_i8,
 * i8_add_bias_sat_dma, i8_element_affine_dma (reference.c of each). */
#define HEXCUDA_ROUND_HALF_AWAY 0
#define HEXCUDA_ROUND_FLOOR 1
int hexcuda_affine_ew(int dev, const void *in, int elem_in, void *out, int elem_out, int64_t n,
                      int32_t zp_in, int32_t mult, int64_t add, int shift, int round, int wrap32,
                      int zp_out, int32_t lo, int32_t hi);
/* KV-cache write: for h < heads, k_cache[h][pos][:] = k_new[h][:] and
 * v_cache[h][pos][:] = v_new[h][:], caches [heads][cache_len][head_dim] int8
 * (kernels/expert/kv_cache_update/reference.c:14-25); 0 <= pos < cache_len. */
int hexcuda_kv_cache_update_i8(int dev, int8_t *k_cache, int8_t *v_cache, const int8_t *k_new,
                               const int8_t *v_new, int pos, int heads, int cache_len,
                               int head_dim);
/* Rotary embedding of interleaved fp16 pairs: out[2p] = x[2p] c - x[2p+1] s,
 * out[2p+1] = x[2p] s + x[2p+1] c with c = cos_t[p], s = sin_t[p], in fp32
 * without fused multiply-adds, one fp16 rounding per output
 * (kernels/expert/rope_pair_fp16/reference.c:5-13).  x and out 4-byte
 * aligned. */
int hexcuda_rope_pair_f16(int dev, const uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                          uint16_t *out, int64_t n_pairs);
/* int8 decoder block: causal LUT-softmax self-attention of X [S][D] (u8)
 * with scores clamp_i8(X.X^T >> 2), h = clamp_u8(X + clamp_i8(P.X >> 8)),
 * then out int8 = sat_i8(h + sat_i8((act_lut[clamp_i8((h.W1 >> 8) + b1) + 128]
 * .W2 >> 7) + b2)); W1 [D][Dff], W2 [Dff][D] int8.
 * kernels/expert/i8_decoder_block/kernel_api.h:53-58. */
/* int8 encoder block (kernels/expert/i8_transformer_encoder_block/
 * reference.c:18-78): self-attention of X [S][D] with itself over every key
 * (query side u8, key / value side the same bytes as int8), scores
 * clamp_i8(sx12 field >> 4), exp-table softmax, h = clamp_u8(X +
 * clamp_i8(sx12 field of P X >> 8)), FFN with H = relu(sx12 field + b1) >> 8
 * (<= 127), out = sat_i8(h + ((sx12 field of H W2 + b2) >> 4)).  One CTA. */
int hexcuda_encoder_block_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut,
                             int8_t *out, int S, int D, int Dff);
int hexcuda_decoder_block_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                             const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                             const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff);

/* s8 x s8 GEMM + fixed-point requant with an optional bias (NULL: none), an
 * optional ReLU between the bias add and the requant and an optional int8
 * residual res [M,N] added with int8 saturation after the requant's clamp;
 * B row-major [K,N] or Bt [N,K].  kernels/expert/gemm_bias_relu_requant/
 * kernel_api.h:14, matmul_residual_add_i8/kernel_api.h; with A = x [1,K] and
 * Bt = the matrix [M,K] it is the matrix-vector form of
 * i8_linear_relu_requant/kernel_api.h:18 and i8_matvec_bias_requant/kernel_api.h:15. */
int hexcuda_gemm_i8_rq_ex(int dev, const int8_t *A, const int8_t *B, int b_transposed,
                          const int32_t *bias, const int8_t *res, int8_t *out, int M, int N,
                          int K, int32_t mult, int shift, int8_t zp, int relu);
/* s8 (a_signed) or u8 A x s8 B GEMM on the raw int32 accumulator: x = acc +
 * bias[j] + res[i][j] in int64 (NULL / HEXCUDA_HMX_RES_NONE: none), then the
 * activation (HEXCUDA_HMX_ACT_*) and the store (HEXCUDA_HMX_STORE_*: I32 /
 * ACC_I32 keep the low 32 bits, I8_SAT / U8_SAT saturate, LUT_I8 reads
 * lut[sat8(x) + 128], LUT_I32 lut[clamp(x + 128, 0, 255)]).  B row-major
 * [K,N] or Bt [N,K].  The int8 GEMM callers gemm_tile_i8, gemm_tile_deepk_i8,
 * i8_gemm_tile, i8_gemm_bias, i8_batch_matmul(_bias), gemm_tile_bias_relu_i8,
 * gemm_bias_gelu, i8_gemm_gelu_lut, ffn_up_gelu_i8 (kernels/expert/<name>/
 * reference.c). */
int hexcuda_gemm_i8_acc(int dev, const void *A, int a_signed, const int8_t *B, int b_transposed,
                        const int32_t *bias, const void *res, int res_kind, const void *lut,
                        void *out, int store, int act, int M, int N, int K);
/* Two-layer int8 FFN: hid = sat8(max(A W1 + b1, 0)) [M,V] (kept on the
 * device), out = sat8(round_half_away((hid W2 + b2) * mult >> shift) + zp)
 * [M,D]; W1 [K,V], W2 [V,D] row-major.  kernels/expert/ffn_relu_block/
 * reference.c. */
int hexcuda_ffn_relu_i8(int dev, const int8_t *A, const int8_t *W1, const int32_t *b1,
                        const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V,
                        int D, int32_t mult, int shift, int8_t zp);
/* Same with a table activation between the layers: hid = act_lut[sat8(A W1 +
 * b1) + 128] (kernels/expert/mlp_block/reference.c:19-30); the second layer
 * and its requant are hexcuda_ffn_relu_i8's. */
int hexcuda_ffn_lut_i8(int dev, const int8_t *A, const int8_t *W1, const int32_t *b1,
                       const int8_t *act_lut, const int8_t *W2, const int32_t *b2, int8_t *out,
                       int M, int K, int V, int D, int32_t mult, int shift, int8_t zp);
/* int16 GEMM: C [M,N] int32 = A [M,K] B [K,N] (int16 row-major), the
 * accumulator modulo 2^32 (kernels/expert/i16_gemm/reference.c:2-11).  The
 * operands are split into signed bytes and multiplied by one tcgen05
 * kind::i8 GEMM of twice the rows and columns; 16 M N bytes of scratch. */
int hexcuda_gemm_i16(int dev, const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K);
/* HMX-convention convolution of in [c_in][ih][iw] (u8) by W
 * [c_out][c_in][kh][kw] (int8) at the given stride, no padding: acc over the
 * window, v = sx12((acc * 17 + 8) >> 4) (+ bias[co]), activation
 * (HEXCUDA_HMX_ACT_*), store HEXCUDA_HMX_STORE_U16_FIELD / I32 / I8_SAT into
 * out [c_out][oh][ow].  Window matrix + HMX GEMM with a column-major store.
 * kernels/expert/i8_conv2d_3x3_hmx, i8_conv2d_3x3_hmx_tiled,
 * i8_conv2d_bias_relu_hmx, i8_conv1d_bias_requant_hmx (ih = kh = 1)
 * reference.c. */
int hexcuda_conv2d_hmx(int dev, const uint8_t *in, const int8_t *W, const int32_t *bias, void *out,
                       int store, int act, int c_in, int ih, int iw, int c_out, int kh, int kw,
                       int stride);
/* Channel-mixing MLP: q = sat_i8(round_half_away((X W1^T + b1) mult1 >>
 * shift1)), y = lut ? lut[q + 128] : q, out = sat_i8(round_half_away((y W2^T
 * + b2) mult2 >> shift2)); X [M,K], W1 [V,K], W2 [D,V] int8 row-major.
 * kernels/expert/i8_channel_mix_block/reference.c:17-40. */
int hexcuda_mix_mlp_i8(int dev, const int8_t *X, const int8_t *W1, const int32_t *b1,
                       const int8_t *lut, const int8_t *W2, const int32_t *b2, int8_t *out, int M,
                       int K, int V, int D, int32_t mult1, int shift1, int32_t mult2, int shift2);
/* Token-mixing MLP of X [T,C]: the same two requantised products along the
 * token axis, W [DM,T], b [DM], W2 [T,DM], b2 [T] (computed as the channel
 * MLP of X^T, transposed back).  kernels/expert/i8_token_mix_block/
 * reference.c:17-41. */
int hexcuda_token_mix_i8(int dev, const int8_t *X, const int8_t *W, const int32_t *b,
                         const int8_t *W2, const int32_t *b2, int8_t *out, int T, int C, int DM,
                         int32_t mult1, int shift1, int32_t mult2, int shift2);
/* int8 RNN cell: h_t = tanh_lut[(uint8) sat_i8(round_half_away((b + Wx x +
 * Wh h_prev) mult >> shift) + zp)], Wx [hidden,in_dim], Wh [hidden,hidden]; one
 * matrix-vector product of [Wx | Wh] by [x, h_prev].
 * kernels/expert/rnn_cell_i8/reference.c. */
int hexcuda_rnn_cell_i8(int dev, const int8_t *Wx, const int8_t *Wh, const int32_t *b,
                        const int8_t *x, const int8_t *h_prev, int8_t *h_t, int hidden, int in_dim,
                        int32_t mult, int shift, int8_t zp, const int8_t *tanh_lut);
/* HMX-convention two-layer FFN: X u8 [M,D], W1 [D,Dff], W2 [Dff,D] int8
 * row-major; r = sx12 field of each product;
 * H = (r1 + b1 > 0) ? min((r1 + b1) >> sh1, 127) : 0 (kept on the device),
 * out = sat_i8((r2 + b2) >> sh2).  kernels/expert/i8_ffn_block/
 * reference.c:8-27 (sh1 8, sh2 3). */
int hexcuda_ffn_hmx_i8(int dev, const uint8_t *X, const int8_t *W1, const int32_t *b1,
                       const int8_t *W2, const int32_t *b2, int8_t *out, int M, int D, int Dff,
                       int sh1, int sh2);
/* HMX-convention SwiGLU FFN: g = clamp_i8(sx12 field of X Wg >> sg), u the
 * same with Wu and su, Hu = u8(clamp((silu_lut[g + 128] (as int8) u) >> sh,
 * -zp, zp - 1) + zp), out = sat_i8((sx12 field of Hu Wd + bd) >> so).
 * kernels/expert/i8_ffn_swiglu_block/reference.c:10-34 (sg 2, su 2, sh 10,
 * zp 8, so 3). */
int hexcuda_ffn_swiglu_hmx_i8(int dev, const uint8_t *X, const int8_t *Wg, const int8_t *Wu,
                              const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut,
                              int8_t *out, int M, int D, int Dff, int sg, int su, int sh, int zp,
                              int so);
/* HMX-convention GEMM with s8 A [M,K] and u8 B [K,N] (the weights-by-
 * activations form of the 1x1 convolutions, i8_conv2d_1x1_hmx/kernel_api.h:17,
 * i8_pointwise_conv_hmx/kernel_api.h:16); store kinds as hexcuda_gemm_hmx_ex
 * without the tables. */
int hexcuda_gemm_hmx_s8u8(int dev, const int8_t *A, const uint8_t *B, void *out, int store,
                          int M, int N, int K);

/* fp16 GEMM, fp32 accumulate, one fp16 rounding: out[M,N] = A[M,K] . Bt[N,K]^T
 * (B column-major).  kernels/expert/fp16_attention_qkt_hmx/kernel_api.h:4-20. */
int hexcuda_gemm_f16_nt(int dev, const uint16_t *A, const uint16_t *Bt,
                        uint16_t *out, int M, int N, int K);
/* fp16 GEMM with the corpus's fp16 post-ops, fp32 accumulate:
 *   v = acc [preround ACC: v = (fp16) acc]
 *   v += res[i][j] (fp16 [M,N], may be NULL) + bias[j] (fp16, may be NULL);
 *   preround SUM: v = (fp16) v; activation; v *= scale; out = (fp16) v.
 * Activations RELU, LEAKY, GELU (below), SIGMOID 1 / (1 + exp(-v)), TANH.
 * B row-major [K,N], or Bt [N,K] with b_transposed.  Bundles
 * (kernels/expert/<name>/kernel_api.h): hmx_matmul_fp16_bias (bias),
 * hmx_matmul_fp16_relu (RELU), fp16_matmul_leaky_relu_hmx (preround, LEAKY:
 * v > 0 ? v : v * 0.125), fp16_matmul_gelu_hmx (preround, GELU: 0.5 v (1 +
 * tanh(0.7978845608 (v + 0.044715 v^3)))), hmx_tile_mac_fp16_32 (res = the
 * output's previous contents), qkt_tile_fp16 (preround, scale),
 * hmx_matmul_fp16_32, fp16_matmul_hmx_32x32, fp16_matmul_hmx_deepk,
 * av_tile_fp16 and hmx_conv1x1_fp16 (plain; the last two with Bt). */
#define HEXCUDA_F16_ACT_NONE 0
#define HEXCUDA_F16_ACT_RELU 1
#define HEXCUDA_F16_ACT_LEAKY 2
#define HEXCUDA_F16_ACT_GELU 3
#define HEXCUDA_F16_ACT_SIGMOID 4
#define HEXCUDA_F16_ACT_TANH 5
#define HEXCUDA_F16_PREROUND_NONE 0
#define HEXCUDA_F16_PREROUND_SUM 1   /* round after the residual and bias adds */
#define HEXCUDA_F16_PREROUND_ACC 2   /* round the accumulator before them:
                                      * fp16_matmul_bias_gelu, fp16_matmul_bias_relu,
                                      * fp16_matmul_residual, fp16_matmul_sigmoid,
                                      * fp16_matmul_tanh, ai_fp16_matmul_gelu */
int hexcuda_gemm_f16_ex(int dev, const uint16_t *A, const uint16_t *B, int b_transposed,
                        const uint16_t *bias, const uint16_t *res, uint16_t *out, int act,
                        int preround, float scale, int M, int N, int K);

/* Same with row-major B[K,N].  kernels/expert/hmx_matmul_fp16_deepk/
 * kernel_api.h:4-10 and fp16_attention_av_hmx/kernel_api.h. */
int hexcuda_gemm_f16_nn(int dev, const uint16_t *A, const uint16_t *B,
                        uint16_t *out, int M, int N, int K);

/* fp16 scaled-dot-product attention with fp32 softmax statistics:
 * O = softmax(scale * Q K^T [+ causal mask j <= i]) V per head.
 * Q, O: [BH, SQ, D]; K, V: [BH, SK, D].
 * kernels/expert/fp16_flash_attention_tile/kernel_api.h:4-42 (recurrence
 * :12-27); candidate_kernel header include/kernel_api/attn_f16.h. */
int hexcuda_attn_f16(int dev, const uint16_t *Q, const uint16_t *K,
                     const uint16_t *V, uint16_t *O, int BH, int SQ, int SK,
                     int D, float scale, int causal);

/* One online-softmax update of a query row's (max, sum, acc) state.
 * kernels/expert/online_softmax_step_fp16/kernel_api.h:4-33. */
int hexcuda_online_softmax_step_f16(int dev, const uint16_t *scores,
                                    const uint16_t *V, uint16_t *running_max,
                                    uint16_t *running_sum, uint16_t *acc,
                                    int BLK, int D);

/* ------------------------------------------------------------ diagnostics */
/* Launch a one-CTA kernel whose bounded wait can never be satisfied: it gives
 * up after budget_ms (1..2000), sets the device watchdog word and returns, so
 * the next hexcuda_sync(dev) returns HEXCUDA_ERR_TIMEOUT and the device stays
 * usable.  Exercises the failure path of every tcgen05 kernel's waits without
 * faulting or hanging the GPU. */
int hexcuda_selftest_watchdog(int dev, uint32_t budget_ms);

/* ------------------------------------------------- host-pointer entries */
/* Same operators on HOST buffers (pageable or pinned).  Rows (M, R, or B*H
 * heads) are split into contiguous shards over the initialised devices;
 * per-column / per-feature operands are replicated.  Blocking.  If nobody
 * called hexcuda_init, the first call initialises device 0 only, or devices
 * 0..HEXCUDA_NGPUS-1 when that environment variable is set. */

int hexcuda_host_softmax_f32(const float *x, float *out, int R, int C);
int hexcuda_host_softmax_f16(const uint16_t *x, uint16_t *out, int R, int C);
int hexcuda_host_layernorm_f32(const float *x, const float *gamma, const float *beta,
                               float *out, int R, int C, float eps);
int hexcuda_host_layernorm_f16(const uint16_t *x, const uint16_t *gamma,
                               const uint16_t *beta, uint16_t *out, int R, int C,
                               float eps);
int hexcuda_host_rmsnorm_f16(const uint16_t *x, const uint16_t *gamma,
                             uint16_t *out, int R, int C, float eps);
int hexcuda_host_rmsnorm_gain_f16(const uint16_t *x, const uint16_t *gain, uint16_t *out, int R,
                                  int C, float eps);
int hexcuda_host_rowreduce_f32(const float *x, float *out, int R, int C, int op);
int hexcuda_host_requant_per_channel(const int32_t *a, int8_t *out, int R, int C,
                                     const int32_t *mult, const int *shift, int8_t zp);
int hexcuda_host_requantize_i32_u8(const int32_t *a, uint8_t *out, int64_t n,
                                   int32_t mult, int shift, uint8_t zp);
int hexcuda_host_requant_ew(const void *a, int a_i8, const void *b, int b_kind, void *out,
                            int64_t n, int pre, int64_t pre_c, int32_t mult, int shift,
                            int zp, int sign_of_a, int lo1, int hi1, int lo2, int hi2,
                            const int8_t *lut);
int hexcuda_host_epilogue_bias_i32(const int32_t *acc, const int32_t *bias, int32_t *out,
                                   int R, int C);
int hexcuda_host_relu_i8(const int8_t *x, int8_t *out, int64_t n);
/* out is a HOST pointer here (the result type of the op, as above); the
 * array is split over the devices and the partial results combined. */
int hexcuda_host_reduce_int(const void *a, const void *b, int elem, int64_t n, int op,
                            void *out);
int hexcuda_host_minmax_ew(const void *a, const void *b, int32_t c, int elem, int op,
                           void *out, int64_t n);
int hexcuda_host_group_sum_i8(const int8_t *a, int32_t *out, int64_t g, int w);
int hexcuda_host_group_dot_i8(const int8_t *a, const int8_t *b, int32_t *out, int64_t g, int w);
int hexcuda_host_gate_mul_requant_i8(const int8_t *gate, const int8_t *up, const int8_t *lut,
                                     int8_t *out, int64_t n, int32_t mult, int shift);
int hexcuda_host_ffn_lut_i8(const int8_t *A, const int8_t *W1, const int32_t *b1,
                            const int8_t *act_lut, const int8_t *W2, const int32_t *b2, int8_t *out,
                            int M, int K, int V, int D, int32_t mult, int shift, int8_t zp);
/* on the first device only (a prefix scan) */
int hexcuda_host_scan_max_i8(const int8_t *in, int8_t *out, int64_t n);
int hexcuda_host_head_group_reduce_i8(const int8_t *X, int8_t *Y, int heads, int G, int64_t MN,
                                      int32_t mult, int shift);
/* x has R rows, or xrows rows gathered through idx (idx not NULL) */
int hexcuda_host_layernorm_lut_i8(const int8_t *x, int xrows, const int32_t *idx,
                                  const int8_t *res, int8_t *out, int R, int W,
                                  const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut,
                                  int affine);
int hexcuda_host_layernorm_lut_i16(const int16_t *x, int16_t *out, int R, int C,
                                   const int16_t *gamma, const int16_t *beta,
                                   const uint16_t *inv_lut, int order);
int hexcuda_host_lut_softmax_u8(const int8_t *x, uint8_t *out, int R, int C,
                                const uint8_t *exp_lut, const uint16_t *recip_lut);
int hexcuda_host_lut_softmax_i16(const int16_t *x, int16_t *out, int R, int C,
                                 const uint16_t *exp_lut);
int hexcuda_host_requant_i16(const int32_t *a, int16_t *out, int64_t n, int32_t mult, int shift);
/* one device */
int hexcuda_host_norm_requant_i8(const int8_t *a, int8_t *out, int64_t n, int nch,
                                 const int32_t *nmult, const int *nshift, int32_t mult, int shift,
                                 int zp);
int hexcuda_host_gemm_softmax_u8(const int8_t *A, const int8_t *B, int b_transposed,
                                 const uint8_t *exp_lut, uint8_t *out, int M, int N, int K,
                                 int requant, int32_t mult, int shift);
int hexcuda_host_gelu_ffn_residual_i8(const int8_t *x, const int8_t *W1, const int32_t *b1,
                                      const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2,
                                      const int8_t *x_res, const int8_t *gamma, const int8_t *beta,
                                      const uint8_t *inv_lut, int8_t *out, int M, int K, int V,
                                      int D);
int hexcuda_host_gemm_i8_requant(const int8_t *A, const int8_t *B, int8_t *out,
                                 int M, int N, int K, int32_t mult, int shift,
                                 int8_t zp);
int hexcuda_host_gemm_i8_bias_requant(const int8_t *A, const int8_t *B,
                                      const int32_t *bias, int8_t *out, int M,
                                      int N, int K, int32_t mult, int shift,
                                      int8_t zp);
int hexcuda_host_gemm_i8_zp(const int8_t *A, const int8_t *B, int8_t *out, int M,
                            int N, int K, int32_t zpA, int32_t scale_mult,
                            int scale_shift);
int hexcuda_host_gemm_u8s8_pc(const uint8_t *A, const int8_t *B, const int32_t *bias,
                              uint8_t *out, int M, int N, int K, int32_t zpA,
                              const int32_t *mult, const int *shift, uint8_t zp_out);
int hexcuda_host_gemm_hmx(const uint8_t *A, const int8_t *B, int b_transposed,
                          const int32_t *bias, void *out, int out_kind, int M, int N,
                          int K, int32_t zpA);
int hexcuda_host_gemm_hmx_ex(const uint8_t *A, const int8_t *B, int b_transposed,
                             const int32_t *bias, const void *res, int res_kind,
                             const void *lut, void *out, int store, int act,
                             int col_major, int M, int N, int K, int32_t zpA);
int hexcuda_host_attn_qkt_av_hmx(const uint8_t *Q, const int8_t *K, const int8_t *V,
                                 int32_t *out, int SQ, int SK, int D);
int hexcuda_host_attn_lut_i8(int mode, const void *Q, const int8_t *K, const int8_t *V,
                             const uint8_t *exp_lut, const int8_t *cos_lut,
                             const int8_t *sin_lut, int rot_shift, void *out, int HQ,
                             int HKV, int S, int D, int32_t scale_mult, int scale_shift,
                             int32_t av_mult, int av_shift);
int hexcuda_host_attn_lut_i8_window(const int8_t *Q, const int8_t *K, const int8_t *V,
                                    const uint8_t *exp_lut, int8_t *out, int heads, int S, int D,
                                    int window, int32_t scale_mult, int scale_shift,
                                    int32_t av_mult, int av_shift);
int hexcuda_host_kv_cache_update_i8(int8_t *k_cache, int8_t *v_cache, const int8_t *k_new,
                                    const int8_t *v_new, int pos, int heads, int cache_len,
                                    int head_dim);
int hexcuda_host_rope_pair_f16(const uint16_t *x, const uint16_t *cos_t, const uint16_t *sin_t,
                               uint16_t *out, int64_t n_pairs);
int hexcuda_host_gemm_i16(const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K);
int hexcuda_host_conv2d_hmx(const uint8_t *in, const int8_t *W, const int32_t *bias, void *out,
                            int store, int act, int c_in, int ih, int iw, int c_out, int kh, int kw,
                            int stride);
int hexcuda_host_mix_mlp_i8(const int8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *lut,
                            const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V,
                            int D, int32_t mult1, int shift1, int32_t mult2, int shift2);
int hexcuda_host_token_mix_i8(const int8_t *X, const int8_t *W, const int32_t *b, const int8_t *W2,
                              const int32_t *b2, int8_t *out, int T, int C, int DM, int32_t mult1,
                              int shift1, int32_t mult2, int shift2);
int hexcuda_host_rnn_cell_i8(const int8_t *Wx, const int8_t *Wh, const int32_t *b, const int8_t *x,
                             const int8_t *h_prev, int8_t *h_t, int hidden, int in_dim, int32_t mult,
                             int shift, int8_t zp, const int8_t *tanh_lut);
int hexcuda_host_affine_ew(const void *in, int elem_in, void *out, int elem_out, int64_t n,
                           int32_t zp_in, int32_t mult, int64_t add, int shift, int round,
                           int wrap32, int zp_out, int32_t lo, int32_t hi);
int hexcuda_host_ffn_hmx_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2,
                            const int32_t *b2, int8_t *out, int M, int D, int Dff, int sh1, int sh2);
int hexcuda_host_ffn_swiglu_hmx_i8(const uint8_t *X, const int8_t *Wg, const int8_t *Wu,
                                   const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut,
                                   int8_t *out, int M, int D, int Dff, int sg, int su, int sh,
                                   int zp, int so);
int hexcuda_host_encoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                  const int8_t *W2, const int32_t *b2, const uint8_t *exp_lut,
                                  int8_t *out, int S, int D, int Dff);
int hexcuda_host_decoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                  const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                                  const uint8_t *exp_lut, int8_t *out, int S, int D, int Dff);
int hexcuda_host_gemm_f16_ex(const uint16_t *A, const uint16_t *B, int b_transposed,
                             const uint16_t *bias, const uint16_t *res, uint16_t *out, int act,
                             int preround, float scale, int M, int N, int K);
int hexcuda_host_gemm_i8_rq_ex(const int8_t *A, const int8_t *B, int b_transposed,
                               const int32_t *bias, const int8_t *res, int8_t *out, int M, int N,
                               int K, int32_t mult, int shift, int8_t zp, int relu);
int hexcuda_host_gemm_i8_acc(const void *A, int a_signed, const int8_t *B, int b_transposed,
                             const int32_t *bias, const void *res, int res_kind, const void *lut,
                             void *out, int store, int act, int M, int N, int K);
int hexcuda_host_ffn_relu_i8(const int8_t *A, const int8_t *W1, const int32_t *b1,
                             const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K,
                             int V, int D, int32_t mult, int shift, int8_t zp);
int hexcuda_host_gemm_hmx_s8u8(const int8_t *A, const uint8_t *B, void *out, int store, int M,
                               int N, int K);
int hexcuda_host_gemm_f16_nt(const uint16_t *A, const uint16_t *Bt, uint16_t *out,
                             int M, int N, int K);
int hexcuda_host_gemm_f16_nn(const uint16_t *A, const uint16_t *B, uint16_t *out,
                             int M, int N, int K);
int hexcuda_host_attn_f16(const uint16_t *Q, const uint16_t *K, const uint16_t *V,
                          uint16_t *O, int BH, int SQ, int SK, int D, float scale,
                          int causal);
int hexcuda_host_online_softmax_step_f16(const uint16_t *scores, const uint16_t *V,
                                         uint16_t *running_max, uint16_t *running_sum,
                                         uint16_t *acc, int BLK, int D);

#ifdef __cplusplus
}
#endif
#endif /* HEXCUDA_H */
