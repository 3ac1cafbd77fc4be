/* candidate_kernel for requantize_i32_i8_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/requantize_i32_i8_dma.h"
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp) {
    hexcuda_host_requant_ew(a, 0, NULL, 0, out, n, HEXCUDA_RQ_PRE_A, 0, mult, shift, zp, 0, -128, 127, -128, 127, NULL);
}
