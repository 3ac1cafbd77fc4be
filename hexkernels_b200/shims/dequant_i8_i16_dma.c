/* candidate_kernel for dequant_i8_i16_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/dequant_i8_i16_dma.h"
void candidate_kernel(const int8_t *a, int16_t *out, int n, int8_t zp, int32_t scale, int shift) {
    hexcuda_host_affine_ew(a, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I16, n, zp, scale, 0, shift, HEXCUDA_ROUND_FLOOR, 1, 0, -32768, 32767);
}
