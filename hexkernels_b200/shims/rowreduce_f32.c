/* candidate_kernel for the fp32 row sum / max on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/rowreduce_f32.h"
void candidate_kernel(const float *x, float *out, int R, int C, int op) {
    hexcuda_host_rowreduce_f32(x, out, R, C, op);
}
