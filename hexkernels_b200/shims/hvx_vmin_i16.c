/* candidate_kernel for hvx_vmin_i16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hvx_vmin_i16.h"
void candidate_kernel(const int16_t *a, const int16_t *b, int16_t *out, int n) {
    hexcuda_host_minmax_ew(a, b, 0, HEXCUDA_ELEM_I16, 1, out, n);
}
