/* candidate_kernel for hvx_vradd_i8_reduce on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hvx_vradd_i8_reduce.h"
void candidate_kernel(const int8_t *a, int32_t *out, int g) {
    hexcuda_host_group_sum_i8(a, out, g, 4);
}
