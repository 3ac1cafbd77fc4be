/* candidate_kernel for residual_add_requant on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/residual_add_requant.h"
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp) {
    hexcuda_host_requant_ew(a, 0, b, 1, out, n, HEXCUDA_RQ_PRE_ADD, 0, mult, shift, zp, 0, -128, 127, -128, 127, NULL);
}
