/* candidate_kernel for kv_cache_update on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/kv_cache_update.h"
void candidate_kernel(int8_t *k_cache, int8_t *v_cache, const int8_t *k_new, const int8_t *v_new, int pos, int num_heads, int cache_len, int head_dim) {
    hexcuda_host_kv_cache_update_i8(k_cache, v_cache, k_new, v_new, pos, num_heads, cache_len, head_dim);
}
