/* candidate_kernel for hvx_vrmpy_i8_dot on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hvx_vrmpy_i8_dot.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *out, int g) {
    hexcuda_host_group_dot_i8(a, b, out, g, 4);
}
