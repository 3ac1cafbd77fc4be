/* candidate_kernel of kernels/expert/epilogue_relu_i8/kernel_api.h:13
 * out = max(x, 0) (int8). */
#ifndef HEXCUDA_KAPI_EPILOGUE_RELU_I8_H
#define HEXCUDA_KAPI_EPILOGUE_RELU_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int n);
#endif
