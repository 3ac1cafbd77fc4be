/* candidate_kernel for fp16_layernorm on the B200: one row, eps 1e-3. */
#include "hexcuda.h"
#include "kernel_api/fp16_layernorm.h"
void candidate_kernel(const hvx_hf *x, const hvx_hf *gamma, const hvx_hf *beta, hvx_hf *out,
                      int n) {
    hexcuda_host_layernorm_f16((const uint16_t *)x, (const uint16_t *)gamma,
                               (const uint16_t *)beta, (uint16_t *)out, 1, n, 1e-3f);
}
