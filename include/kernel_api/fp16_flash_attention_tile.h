/* candidate_kernel of kernels/expert/fp16_flash_attention_tile/kernel_api.h:41-42:
 * one head, SQ queries against SK keys/values of width DH, non-causal, scale
 * FLASH_SCALE (0.125, kernel_api.h:39). */
#ifndef HEXCUDA_KAPI_FP16_FLASH_ATTENTION_TILE_H
#define HEXCUDA_KAPI_FP16_FLASH_ATTENTION_TILE_H
#include "hvx_hf.h"
#ifndef FLASH_SCALE
#define FLASH_SCALE 0.125f
#endif
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, const hvx_hf *V,
                      hvx_hf *O, int SQ, int SK, int DH);
#endif
