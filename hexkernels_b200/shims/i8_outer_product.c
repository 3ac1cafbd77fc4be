/* candidate_kernel for i8_outer_product on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_outer_product.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *C, int M, int N) {
    hexcuda_host_gemm_i8_acc(a, 1, b, 0, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, C, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, M, N, 1);
}
