/* candidate_kernel for requant_add_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/requant_add_dma.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n) {
    hexcuda_host_requant_ew(a, 0, b, 1, out, n, HEXCUDA_RQ_PRE_ADD, 0, 5, 3, 0, 0, -128, 127, -128, 127, NULL);
}
