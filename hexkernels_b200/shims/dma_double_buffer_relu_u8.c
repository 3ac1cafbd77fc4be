/* candidate_kernel for dma_double_buffer_relu_u8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/dma_double_buffer_relu_u8.h"
void candidate_kernel(const uint8_t *a, uint8_t *out, int n) {
    hexcuda_host_affine_ew(a, HEXCUDA_ELEM_U8, out, HEXCUDA_ELEM_U8, n, 128, 1, 0, 0, HEXCUDA_ROUND_FLOOR, 1, 0, 0, 255);
}
