/* candidate_kernel for i8_norm_requant_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_norm_requant_dma.h"
/* the task's fixed per-channel tables (i8_norm_requant_dma/reference.c:6-12) */
static const int32_t kNormMult[16] = {3, 5, 7, 9, 11, 13, 15, 17, 3, 5, 7, 9, 11, 13, 15, 17};
static const int kNormShift[16] = {2, 3, 4, 5, 3, 4, 5, 6, 2, 3, 4, 5, 3, 4, 5, 6};
void candidate_kernel(const int8_t *a, int8_t *out, int n) {
    hexcuda_host_norm_requant_i8(a, out, n, 16, kNormMult, kNormShift, 5, 4, 0);
}
