/* candidate_kernel of kernels/expert/i8_attention_av_hmx/kernel_api.h:16
 * out[i][d] = unsigned 12-bit HMX field of sum_j P[i][j] V[j][d] (uint16). */
#ifndef HEXCUDA_KAPI_I8_ATTENTION_AV_HMX_H
#define HEXCUDA_KAPI_I8_ATTENTION_AV_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *P, const int8_t *V, uint16_t *out, int S, int D);
#endif
