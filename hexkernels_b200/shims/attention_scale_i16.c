/* candidate_kernel for attention_scale_i16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/attention_scale_i16.h"
void candidate_kernel(const int32_t *raw, int16_t *out, int M, int N, int32_t scale_mult, int scale_shift) {
    hexcuda_host_requant_i16(raw, out, (int64_t)M * N, scale_mult, scale_shift);
}
