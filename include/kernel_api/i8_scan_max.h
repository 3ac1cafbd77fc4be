/* candidate_kernel of kernels/expert/i8_scan_max/kernel_api.h:7
 * inclusive prefix maximum of int8. */
#ifndef HEXCUDA_KAPI_I8_SCAN_MAX_H
#define HEXCUDA_KAPI_I8_SCAN_MAX_H
#include <stdint.h>
void candidate_kernel(const int8_t *in, int8_t *out, int n);
#endif
