/* candidate_kernel for embedding_layer_norm on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/embedding_layer_norm.h"
void candidate_kernel(const int8_t *table, const int32_t *idx, int8_t *out, int T, int D, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut) {
    int rows = 1;
    for (int i = 0; i < T; i++)
        if (idx[i] + 1 > rows) rows = idx[i] + 1;
    hexcuda_host_layernorm_lut_i8(table, rows, idx, NULL, out, T, D, gamma, beta, inv_lut, HEXCUDA_LN_AFFINE_SHARED);
}
