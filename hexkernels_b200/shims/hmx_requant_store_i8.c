/* candidate_kernel for hmx_requant_store_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hmx_requant_store_i8.h"
void candidate_kernel(const int32_t *acc, int8_t *out, int n) {
    hexcuda_host_affine_ew(acc, HEXCUDA_ELEM_I32, out, HEXCUDA_ELEM_I8, n, 0, 17, 8, 4, HEXCUDA_ROUND_FLOOR, 1, 0, -128, 127);
}
