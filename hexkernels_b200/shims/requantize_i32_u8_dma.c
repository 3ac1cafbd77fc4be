/* candidate_kernel for requantize_i32_u8_dma on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/requantize_i32_u8_dma.h"
void candidate_kernel(const int32_t *a, uint8_t *out, int n, int32_t mult, int shift,
                      uint8_t zp) {
    hexcuda_host_requantize_i32_u8(a, out, n, mult, shift, zp);
}
