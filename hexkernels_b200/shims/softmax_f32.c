/* candidate_kernel for the fp32 row softmax on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/softmax_f32.h"
void candidate_kernel(const float *x, float *out, int R, int C) {
    hexcuda_host_softmax_f32(x, out, R, C);
}
