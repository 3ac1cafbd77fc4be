/* candidate_kernel for mul_add_requant_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/mul_add_requant_dma.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n) {
    hexcuda_host_requant_ew(a, 0, b, 1, out, n, HEXCUDA_RQ_PRE_MUL_ADD, 50, 3, 1, 0, 0, -128, 127, -128, 127, NULL);
}
