/* candidate_kernel for i8_matvec_bias_requant on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_matvec_bias_requant.h"
void candidate_kernel(const int8_t *A, const int8_t *x, const int32_t *bias, int8_t *out, int M, int K, int32_t mult, int shift, int8_t zp) {
    hexcuda_host_gemm_i8_rq_ex(x, A, 1, bias, NULL, out, 1, M, K, mult, shift, zp, 0);
}
