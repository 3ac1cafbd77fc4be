/* candidate_kernel for i8_conv2d_3x3_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_conv2d_3x3_hmx.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n) {
    (void)n;
    hexcuda_host_conv2d_hmx(in, W, NULL, out, HEXCUDA_HMX_STORE_U16_FIELD, HEXCUDA_HMX_ACT_NONE, 8, 10, 10, 32, 3, 3, 1);
}
