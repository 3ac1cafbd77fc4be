/* candidate_kernel for requant_per_channel on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/requant_per_channel.h"
void candidate_kernel(const int32_t *a, int8_t *out, int R, int C,
                      const int32_t *mult, const int *shift, int8_t zp) {
    hexcuda_host_requant_per_channel(a, out, R, C, mult, shift, zp);
}
