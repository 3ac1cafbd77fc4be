/* candidate_kernel of kernels/expert/i8_chunk_norm/kernel_api.h:28
 * int8 layernorm over G chunks of n / G elements, per-chunk gamma / beta segments. */
#ifndef HEXCUDA_KAPI_I8_CHUNK_NORM_H
#define HEXCUDA_KAPI_I8_CHUNK_NORM_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int n, int G, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut);
#endif
