/* candidate_kernel for hmx_kacc_i8_4tile on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hmx_kacc_i8_4tile.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n, int K) {
    hexcuda_host_gemm_hmx_ex(A, B, 0, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 0, n, n, K, 0);
}
