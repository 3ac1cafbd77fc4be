/* candidate_kernel for u8_clamp_range_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/u8_clamp_range_dma.h"
void candidate_kernel(const uint8_t *in, uint8_t *out, int n) {
    hexcuda_host_affine_ew(in, HEXCUDA_ELEM_U8, out, HEXCUDA_ELEM_U8, n, 0, 1, 0, 0, HEXCUDA_ROUND_FLOOR, 1, 0, 64, 191);
}
