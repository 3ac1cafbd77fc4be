/* candidate_kernel of kernels/expert/residual_add_requant/kernel_api.h:12
 * elementwise requant: pre add, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_RESIDUAL_ADD_REQUANT_H
#define HEXCUDA_KAPI_RESIDUAL_ADD_REQUANT_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp);
#endif
