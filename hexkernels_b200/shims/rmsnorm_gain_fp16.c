/* candidate_kernel for rmsnorm_gain_fp16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/rmsnorm_gain_fp16.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *x, const hvx_hf *gain, hvx_hf *out, int R, int C) {
    hexcuda_host_rmsnorm_gain_f16(U(x), U(gain), W(out), R, C, 1e-3f);
}
