/* candidate_kernel of kernels/expert/gemm_tile_zp_i8/kernel_api.h:26-28:
 * acc = A.B - zpA * colsum(B) (int32), out = sat_i8(round_half_away(acc *
 * scale_mult >> scale_shift)). */
#ifndef HEXCUDA_KAPI_GEMM_TILE_ZP_I8_H
#define HEXCUDA_KAPI_GEMM_TILE_ZP_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out,
                      int M, int N, int K,
                      int32_t zpA, int32_t scale_mult, int scale_shift);
#endif
