/* candidate_kernel for vtcm_reduce_i32 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/vtcm_reduce_i32.h"
void candidate_kernel(const int32_t *a, int n, int32_t *out) {
    hexcuda_host_reduce_int(a, NULL, HEXCUDA_ELEM_I32, n, HEXCUDA_RED_SUM, out);
}
