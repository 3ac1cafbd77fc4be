/* candidate_kernel of kernels/expert/av_tile_fp16/kernel_api.h:23
 * O = A V^T with V stored [D][N]. */
#ifndef HEXCUDA_KAPI_AV_TILE_FP16_H
#define HEXCUDA_KAPI_AV_TILE_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *V, hvx_hf *O, int M, int N, int D);
#endif
