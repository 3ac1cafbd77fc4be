/* candidate_kernel of kernels/expert/mlp_gate_silu_i8/kernel_api.h:22
 * SiLU-table gate times up, round-half-away requant, int8 out. */
#ifndef HEXCUDA_KAPI_MLP_GATE_SILU_I8_H
#define HEXCUDA_KAPI_MLP_GATE_SILU_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *gate, const int8_t *up, const int8_t *silu_lut, int8_t *out, int N, int32_t scale_mult, int scale_shift);
#endif
