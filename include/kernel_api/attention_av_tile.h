/* candidate_kernel of kernels/expert/attention_av_tile/kernel_api.h:19
 * int8 A V (V [N,D]), int32 out. */
#ifndef HEXCUDA_KAPI_ATTENTION_AV_TILE_H
#define HEXCUDA_KAPI_ATTENTION_AV_TILE_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *V, int32_t *O, int M, int N, int D);
#endif
