/* New task header: per-row reduction of an R x C fp32 matrix into out[R];
 * op 0 = sum (kernels/mined/fp32_sum/reference.c:8-14 per row), op 1 = max. */
#ifndef HEXCUDA_KAPI_ROWREDUCE_F32_H
#define HEXCUDA_KAPI_ROWREDUCE_F32_H
void candidate_kernel(const float *x, float *out, int R, int C, int op);
#endif
