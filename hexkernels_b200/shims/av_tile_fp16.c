/* candidate_kernel for av_tile_fp16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/av_tile_fp16.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
#define W_(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *A, const hvx_hf *V, hvx_hf *O, int M, int N, int D) {
    hexcuda_host_gemm_f16_ex(U(A), U(V), 1, NULL, NULL, W(O), HEXCUDA_F16_ACT_NONE, 0, 1.0f, M, D, N);
}
