/* candidate_kernel for i8_sparse_attn_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_sparse_attn_block.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut, int8_t *out, int window, int32_t smult, int sshift, int32_t amult, int ashift) {
    hexcuda_host_attn_lut_i8_window(Q, K, V, exp_lut, out, SPARSE_ATTN_H, SPARSE_ATTN_SEQ, SPARSE_ATTN_HEAD_DIM, window, smult, sshift, amult, ashift);
}
