/* New task header (no corpus bundle has it): the fp32 variant of
 * kernels/expert/fp16_softmax/kernel_api.h:15 for the 65536 x 4096 fp32
 * row-softmax benchmark case.  Row softmax over the last axis:
 *   out[r][j] = expf(x[r][j] - max_j x[r]) / sum_j expf(x[r][j] - max_j x[r]). */
#ifndef HEXCUDA_KAPI_SOFTMAX_F32_H
#define HEXCUDA_KAPI_SOFTMAX_F32_H
void candidate_kernel(const float *x, float *out, int R, int C);
#endif
