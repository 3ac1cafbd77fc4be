/* candidate_kernel for i8_gqa_qkt_hmx backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, uint16_t *out) {
    for (int hq = 0; hq < GQA_H_Q; hq++)
        oracle_gemm_hmx_ex_rows(Q + (size_t)hq * GQA_S * GQA_D, K + (size_t)(hq / GQA_GROUP_SIZE) * GQA_S * GQA_D, 1,
                                out + (size_t)hq * GQA_S * GQA_S, GQA_S, GQA_S, GQA_D, 0, ORACLE_HMX_STORE_U16_FIELD,
                                ORACLE_HMX_ACT_NONE, NULL, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, GQA_S);
}
