/* New task header: kernels/expert/fp16_layernorm/kernel_api.h:4-18 applied to
 * every row of an R x C fp32 matrix, eps a parameter (the corpus hardwires
 * 1e-3):  mean = sum x / C; var = max(sum x^2 / C - mean^2, 0);
 *         out = (x - mean) / sqrtf(var + eps) * gamma[j] + beta[j]. */
#ifndef HEXCUDA_KAPI_LAYERNORM_F32_H
#define HEXCUDA_KAPI_LAYERNORM_F32_H
void candidate_kernel(const float *x, const float *gamma, const float *beta,
                      float *out, int R, int C, float eps);
#endif
