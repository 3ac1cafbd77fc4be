/* candidate_kernel of kernels/expert/hmx_requant_store_i8/kernel_api.h:13
 * (acc * 17 + 8) >> 4 in int32, int8 saturation. */
#ifndef HEXCUDA_KAPI_HMX_REQUANT_STORE_I8_H
#define HEXCUDA_KAPI_HMX_REQUANT_STORE_I8_H
#include <stdint.h>
void candidate_kernel(const int32_t *acc, int8_t *out, int n);
#endif
