/* candidate_kernel of kernels/expert/embedding_layer_norm/kernel_api.h:28
 * embedding gather (table rows idx[i]) and int8 layernorm. */
#ifndef HEXCUDA_KAPI_EMBEDDING_LAYER_NORM_H
#define HEXCUDA_KAPI_EMBEDDING_LAYER_NORM_H
#include <stdint.h>
void candidate_kernel(const int8_t *table, const int32_t *idx, int8_t *out, int T, int D, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut);
#endif
