/* candidate_kernel for i8_attention_qkt_av_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_attention_qkt_av_hmx.h"
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      int32_t *out, int S, int D) {
    hexcuda_host_attn_qkt_av_hmx(Q, K, V, out, S, S, D);
}
