/* candidate_kernel of kernels/expert/i8_attention_qkt_av_hmx/kernel_api.h:19
 * out = sx12 field of (sx12 field of Q K^T) V (int32). */
#ifndef HEXCUDA_KAPI_I8_ATTENTION_QKT_AV_HMX_H
#define HEXCUDA_KAPI_I8_ATTENTION_QKT_AV_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      int32_t *out, int S, int D);
#endif
