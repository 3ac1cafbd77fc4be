/* candidate_kernel of kernels/expert/i8_attention_qkt_hmx/kernel_api.h:16
 * scores out[i][j] = unsigned 12-bit HMX field of sum_d Q[i][d] K[j][d] (uint16). */
#ifndef HEXCUDA_KAPI_I8_ATTENTION_QKT_HMX_H
#define HEXCUDA_KAPI_I8_ATTENTION_QKT_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *Q, const int8_t *K, uint16_t *out, int S, int D);
#endif
