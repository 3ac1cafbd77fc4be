/* candidate_kernel for epilogue_bias_i32 on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/epilogue_bias_i32.h"
void candidate_kernel(const int32_t *acc, const int32_t *bias, int32_t *out, int R, int C) {
    hexcuda_host_epilogue_bias_i32(acc, bias, out, R, C);
}
