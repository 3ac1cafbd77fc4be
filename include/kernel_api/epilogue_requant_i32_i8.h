/* candidate_kernel of kernels/expert/epilogue_requant_i32_i8/kernel_api.h:19
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_EPILOGUE_REQUANT_I32_I8_H
#define HEXCUDA_KAPI_EPILOGUE_REQUANT_I32_I8_H
#include <stdint.h>
void candidate_kernel(const int32_t *acc, int8_t *out, int n, int32_t mult, int shift);
#endif
