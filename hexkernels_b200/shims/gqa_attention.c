/* candidate_kernel for gqa_attention on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/gqa_attention.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut,
                      int8_t *out, int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift) {
    hexcuda_host_attn_lut_i8(HEXCUDA_ATTN_LUT_REQUANT, Q, K, V, exp_lut, NULL, NULL, 0, out, H_Q, H_KV, SEQ, HEAD_DIM, scale_mult, scale_shift, av_mult, av_shift);
}
