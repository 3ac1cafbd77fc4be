/* candidate_kernel of kernels/expert/av_tile_i8/kernel_api.h:25
 * int8 A V^T (V [D,N]), int32 out. */
#ifndef HEXCUDA_KAPI_AV_TILE_I8_H
#define HEXCUDA_KAPI_AV_TILE_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *V, int32_t *O, int M, int N, int D);
#endif
