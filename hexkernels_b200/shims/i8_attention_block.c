/* candidate_kernel for i8_attention_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_attention_block.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      uint16_t *out, int S, int D, const uint8_t *exp_lut) {
    hexcuda_host_attn_lut_i8(HEXCUDA_ATTN_LUT_HMX, Q, K, V, exp_lut, NULL, NULL, 0, out, 1, 1, S, D, 0, 0, 0, 0);
}
