/* candidate_kernel of kernels/expert/hmx_tile_mac_fp16_32/kernel_api.h:11
 * out += A B (fp32 accumulate from the old out, one fp16 rounding). */
#ifndef HEXCUDA_KAPI_HMX_TILE_MAC_FP16_32_H
#define HEXCUDA_KAPI_HMX_TILE_MAC_FP16_32_H
#include "hvx_hf.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n);
#endif
