/* candidate_kernel for i8_attention_qkt_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_attention_qkt_hmx.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, uint16_t *out, int S, int D) {
    hexcuda_host_gemm_hmx_ex(Q, K, 1, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_U16_FIELD, HEXCUDA_HMX_ACT_NONE, 0, S, S, D, 0);
}
