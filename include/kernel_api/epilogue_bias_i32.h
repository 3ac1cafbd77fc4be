/* candidate_kernel of kernels/expert/epilogue_bias_i32/kernel_api.h:14
 * out[r][c] = acc[r][c] + bias[c] (int32). */
#ifndef HEXCUDA_KAPI_EPILOGUE_BIAS_I32_H
#define HEXCUDA_KAPI_EPILOGUE_BIAS_I32_H
#include <stdint.h>
void candidate_kernel(const int32_t *acc, const int32_t *bias, int32_t *out, int R, int C);
#endif
