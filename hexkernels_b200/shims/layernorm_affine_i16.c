/* candidate_kernel for layernorm_affine_i16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/layernorm_affine_i16.h"
void candidate_kernel(const int16_t *x, int16_t *out, int R, int C, const int16_t *gamma, const int16_t *beta, const uint16_t *inv_lut) {
    hexcuda_host_layernorm_lut_i16(x, out, R, C, gamma, beta, inv_lut, 1);
}
