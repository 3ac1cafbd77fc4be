/* candidate_kernel for qkt_tile_fp16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/qkt_tile_fp16.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
#define W_(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *S, int M, int N, int D, _Float16 scale) {
    hexcuda_host_gemm_f16_ex(U(Q), U(K), 0, NULL, NULL, W(S), HEXCUDA_F16_ACT_NONE, 1, (float)scale, M, N, D);
}
