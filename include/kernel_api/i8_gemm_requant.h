/* candidate_kernel of kernels/expert/i8_gemm_requant/kernel_api.h:9-11.
 * out = sat_i8(round_half_away((int64)(A.B) * mult >> shift) + zp);
 * A [M,K] s8, B [K,N] s8 row-major.  Also the int8 x int8 -> int32 GEMM
 * M=N=K=256 benchmark case. */
#ifndef HEXCUDA_KAPI_I8_GEMM_REQUANT_H
#define HEXCUDA_KAPI_I8_GEMM_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out,
                      int M, int N, int K, int32_t mult, int shift, int8_t zp);
#endif
