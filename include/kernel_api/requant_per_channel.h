/* candidate_kernel of kernels/expert/requant_per_channel/kernel_api.h:10-11:
 * row r of the R x C int32 input uses mult[r], shift[r]; shared zp; int8. */
#ifndef HEXCUDA_KAPI_REQUANT_PER_CHANNEL_H
#define HEXCUDA_KAPI_REQUANT_PER_CHANNEL_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int R, int C,
                      const int32_t *mult, const int *shift, int8_t zp);
#endif
