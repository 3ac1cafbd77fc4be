/* candidate_kernel for i8_scan_max on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_scan_max.h"
void candidate_kernel(const int8_t *in, int8_t *out, int n) {
    hexcuda_host_scan_max_i8(in, out, n);
}
