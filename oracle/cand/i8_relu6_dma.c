/* candidate_kernel for i8_relu6_dma backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n, int8_t scale) {
    /* cap = (int8)(6 scale) as the reference computes it.  cap >= 0: the
     * clamp of x to [0, cap].  A wrapped cap < 0 sends x < 0 to 0 and
     * x >= 0 to cap, which is the clamp of -1000 x + cap to [cap, 0]. */
    const int cap = (int8_t)(6 * (int)scale);
    if (cap >= 0)
        oracle_affine_ew(x, ORACLE_ELEM_I8, out, ORACLE_ELEM_I8, n, 0, 1, 0, 0, 1, 1, 0, 0, cap);
    else
        oracle_affine_ew(x, ORACLE_ELEM_I8, out, ORACLE_ELEM_I8, n, 0, -1000, cap, 0, 1, 1, 0, cap, 0);
}
