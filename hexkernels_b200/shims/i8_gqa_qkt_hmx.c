/* candidate_kernel for i8_gqa_qkt_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_gqa_qkt_hmx.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, uint16_t *out) {
    for (int hq = 0; hq < GQA_H_Q; hq++)
        hexcuda_host_gemm_hmx_ex(Q + (size_t)hq * GQA_S * GQA_D, K + (size_t)(hq / GQA_GROUP_SIZE) * GQA_S * GQA_D,
                                 1, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, out + (size_t)hq * GQA_S * GQA_S,
                                 HEXCUDA_HMX_STORE_U16_FIELD, HEXCUDA_HMX_ACT_NONE, 0, GQA_S, GQA_S, GQA_D, 0);
}
