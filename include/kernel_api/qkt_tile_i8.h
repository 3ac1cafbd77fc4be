/* candidate_kernel of kernels/expert/qkt_tile_i8/kernel_api.h:30
 * int8 Q K (K [D,N]) requantised to int8. */
#ifndef HEXCUDA_KAPI_QKT_TILE_I8_H
#define HEXCUDA_KAPI_QKT_TILE_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *Q, const int8_t *K, int8_t *S, int M, int N, int D, int32_t scale_mult, int scale_shift);
#endif
