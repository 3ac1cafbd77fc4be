// attn_tc.cu -- tcgen05 flash-attention path (placeholder: shapes are routed
// to the CUDA-core path in attn.cu until this kernel is enabled).
#include <cuda_fp16.h>

#include "hx_internal.h"

namespace hx {

int attn_tc_launch(Dev *, const __half *, const __half *, const __half *, __half *, int, int, int,
                   int, float, int, bool *handled) {
    *handled = false;
    return HEXCUDA_OK;
}

}  // namespace hx
