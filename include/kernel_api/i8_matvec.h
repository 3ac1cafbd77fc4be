/* candidate_kernel of kernels/expert/i8_matvec/kernel_api.h:7
 * int8 matrix-vector product, int32 out. */
#ifndef HEXCUDA_KAPI_I8_MATVEC_H
#define HEXCUDA_KAPI_I8_MATVEC_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *x, int32_t *y, int M, int K);
#endif
