/* candidate_kernel for epilogue_relu_i8 on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/epilogue_relu_i8.h"
void candidate_kernel(const int8_t *x, int8_t *out, int n) {
    hexcuda_host_relu_i8(x, out, n);
}
