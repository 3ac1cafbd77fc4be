/* candidate_kernel of kernels/expert/attention_qkt_tile/kernel_api.h:25
 * int8 Q K^T (K [N,D]) requantised to int8. */
#ifndef HEXCUDA_KAPI_ATTENTION_QKT_TILE_H
#define HEXCUDA_KAPI_ATTENTION_QKT_TILE_H
#include <stdint.h>
void candidate_kernel(const int8_t *Q, const int8_t *K, int8_t *S, int M, int N, int D, int32_t scale_mult, int scale_shift);
#endif
