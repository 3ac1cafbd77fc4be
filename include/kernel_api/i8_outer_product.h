/* candidate_kernel of kernels/expert/i8_outer_product/kernel_api.h:6
 * int8 outer product (a GEMM with K = 1), int32 out. */
#ifndef HEXCUDA_KAPI_I8_OUTER_PRODUCT_H
#define HEXCUDA_KAPI_I8_OUTER_PRODUCT_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *C, int M, int N);
#endif
