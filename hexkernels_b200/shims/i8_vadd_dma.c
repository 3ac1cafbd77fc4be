/* candidate_kernel for i8_vadd_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_vadd_dma.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n) {
    hexcuda_host_requant_ew(a, 1, b, 2, out, n, HEXCUDA_RQ_PRE_ADD, 0, 1, 0, 0, 0, -256, 255, -256, 255, NULL);
}
