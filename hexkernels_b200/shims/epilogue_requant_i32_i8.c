/* candidate_kernel for epilogue_requant_i32_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/epilogue_requant_i32_i8.h"
void candidate_kernel(const int32_t *acc, int8_t *out, int n, int32_t mult, int shift) {
    hexcuda_host_requant_ew(acc, 0, NULL, 0, out, n, HEXCUDA_RQ_PRE_A, 0, mult, shift, 0, 0, -128, 127, -128, 127, NULL);
}
