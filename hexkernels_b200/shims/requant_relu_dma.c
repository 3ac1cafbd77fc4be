/* candidate_kernel for requant_relu_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/requant_relu_dma.h"
void candidate_kernel(const int32_t *a, int8_t *out, int n) {
    hexcuda_host_requant_ew(a, 0, NULL, 0, out, n, HEXCUDA_RQ_PRE_A, 0, 13, 3, 0, 0, 0, 127, 0, 127, NULL);
}
