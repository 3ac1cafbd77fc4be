/* New task header for batched, optionally causal fp16 attention (the B=8,
 * H=32, S=4096, D=128 benchmark case).  Generalises
 * kernels/expert/fp16_flash_attention_tile/kernel_api.h:12-42 (one head,
 * hardwired FLASH_SCALE, SK <= 64) to B*H heads of [S, D] Q/K/V/O, a scale
 * parameter and a causal window (key j visible to query i iff j <= i):
 *   O[b,h,i,:] = sum_j softmax_j(scale * Q[b,h,i,:] . K[b,h,j,:]) V[b,h,j,:]
 * with fp32 scores and softmax statistics, fp16 out. */
#ifndef HEXCUDA_KAPI_ATTN_F16_H
#define HEXCUDA_KAPI_ATTN_F16_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, const hvx_hf *V,
                      hvx_hf *O, int B, int H, int S, int D, float scale,
                      int causal);
#endif
