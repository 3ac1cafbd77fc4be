/* candidate_kernel of kernels/expert/i8_gemm_bias_requant/kernel_api.h:15-18:
 * the requant of i8_gemm_requant applied to (int64)acc + bias[j]. */
#ifndef HEXCUDA_KAPI_I8_GEMM_BIAS_REQUANT_H
#define HEXCUDA_KAPI_I8_GEMM_BIAS_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B,
                      const int32_t *bias, int8_t *out,
                      int M, int N, int K,
                      int32_t mult, int shift, int8_t zp);
#endif
