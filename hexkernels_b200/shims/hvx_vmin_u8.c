/* candidate_kernel for hvx_vmin_u8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hvx_vmin_u8.h"
void candidate_kernel(const uint8_t *a, const uint8_t *b, uint8_t *out, int n) {
    hexcuda_host_minmax_ew(a, b, 0, HEXCUDA_ELEM_U8, 1, out, n);
}
