/* candidate_kernel for rope_pair_fp16 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/rope_pair_fp16.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *x, const hvx_hf *cos, const hvx_hf *sin, hvx_hf *out, int n_pairs) {
    hexcuda_host_rope_pair_f16(U(x), U(cos), U(sin), W(out), n_pairs);
}
