/* candidate_kernel for batched causal/non-causal fp16 attention on the B200:
 * the B*H heads are sharded over the initialised devices. */
#include "hexcuda.h"
#include "kernel_api/attn_f16.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, const hvx_hf *V, hvx_hf *O, int B, int H,
                      int S, int D, float scale, int causal) {
    hexcuda_host_attn_f16((const uint16_t *)Q, (const uint16_t *)K, (const uint16_t *)V,
                          (uint16_t *)O, B * H, S, S, D, scale, causal);
}
