/* candidate_kernel of kernels/expert/qkt_tile_fp16/kernel_api.h:33
 * S = (fp16)((fp16)(Q K) * scale), K stored [D][N]. */
#ifndef HEXCUDA_KAPI_QKT_TILE_FP16_H
#define HEXCUDA_KAPI_QKT_TILE_FP16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *S, int M, int N, int D, _Float16 scale);
#endif
