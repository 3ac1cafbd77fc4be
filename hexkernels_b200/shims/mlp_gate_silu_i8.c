/* candidate_kernel for mlp_gate_silu_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/mlp_gate_silu_i8.h"
void candidate_kernel(const int8_t *gate, const int8_t *up, const int8_t *silu_lut, int8_t *out, int N, int32_t scale_mult, int scale_shift) {
    hexcuda_host_gate_mul_requant_i8(gate, up, silu_lut, out, N, scale_mult, scale_shift);
}
