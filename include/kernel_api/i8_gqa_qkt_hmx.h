/* candidate_kernel of kernels/expert/i8_gqa_qkt_hmx/kernel_api.h:30
 * per query head hq: out[hq] = unsigned 12-bit field of Q[hq] K[hq / GQA_GROUP_SIZE]^T. */
#ifndef HEXCUDA_KAPI_I8_GQA_QKT_HMX_H
#define HEXCUDA_KAPI_I8_GQA_QKT_HMX_H
#include <stdint.h>
/* the task's fixed shape (its kernel_api.h:24-28) */
#define GQA_H_Q 2
#define GQA_H_KV 1
#define GQA_GROUP_SIZE 2
#define GQA_S 64
#define GQA_D 64
void candidate_kernel(const uint8_t *Q, const int8_t *K, uint16_t *out);
#endif
