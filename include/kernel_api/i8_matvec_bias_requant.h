/* candidate_kernel of kernels/expert/i8_matvec_bias_requant/kernel_api.h:15
 * y = A x + bias, requant (A [M][K]); run as the 1-row GEMM x^T A^T. */
#ifndef HEXCUDA_KAPI_I8_MATVEC_BIAS_REQUANT_H
#define HEXCUDA_KAPI_I8_MATVEC_BIAS_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *x, const int32_t *bias, int8_t *out, int M, int K, int32_t mult, int shift, int8_t zp);
#endif
