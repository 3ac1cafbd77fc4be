/* candidate_kernel for i8_pointwise_conv_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_pointwise_conv_hmx.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n) {
    (void)n;
    hexcuda_host_gemm_hmx_s8u8(W, in, out, HEXCUDA_HMX_STORE_U16_FIELD, CONV_COUT, CONV_P, CONV_CIN);
}
