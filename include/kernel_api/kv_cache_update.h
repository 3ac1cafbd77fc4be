/* candidate_kernel of kernels/expert/kv_cache_update/kernel_api.h:24
 * int8 KV-cache row write at position pos for every head. */
#ifndef HEXCUDA_KAPI_KV_CACHE_UPDATE_H
#define HEXCUDA_KAPI_KV_CACHE_UPDATE_H
#include <stdint.h>
void candidate_kernel(int8_t *k_cache, int8_t *v_cache, const int8_t *k_new, const int8_t *v_new, int pos, int num_heads, int cache_len, int head_dim);
#endif
