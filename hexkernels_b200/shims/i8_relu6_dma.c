/* candidate_kernel for i8_relu6_dma on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_relu6_dma.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n, int8_t scale) {
    /* cap = (int8)(6 scale) as the reference computes it.  cap >= 0: the
     * clamp of x to [0, cap].  A wrapped cap < 0 sends x < 0 to 0 and
     * x >= 0 to cap, which is the clamp of -1000 x + cap to [cap, 0]. */
    const int cap = (int8_t)(6 * (int)scale);
    if (cap >= 0)
        hexcuda_host_affine_ew(x, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, 1, 0, 0, HEXCUDA_ROUND_FLOOR, 1, 0, 0, cap);
    else
        hexcuda_host_affine_ew(x, HEXCUDA_ELEM_I8, out, HEXCUDA_ELEM_I8, n, 0, -1000, cap, 0, HEXCUDA_ROUND_FLOOR, 1, 0, cap, 0);
}
