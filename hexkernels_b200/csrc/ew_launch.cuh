// ew_launch.cuh -- grid size of the grid-stride streaming kernels.
#pragma once
#include "hx_internal.h"

namespace hx {

// Enough 256-thread blocks for `work` thread steps, capped at what the device
// keeps resident at once (blocks per SM from the kernel's register and
// shared-memory use, cached per kernel and device), so every block runs in
// the first and only wave.
template <auto KERN>
int resident_blocks(const Dev *d, int64_t work) {
    static int per_sm[64] = {};
    const int slot = d->ordinal & 63;
    if (per_sm[slot] == 0) {
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, KERN, 256, 0) != cudaSuccess || nb < 1) {
            cudaGetLastError();
            nb = 1;
        }
        per_sm[slot] = nb;
    }
    int64_t blocks = (work + 255) / 256;
    const int64_t cap = (int64_t)d->sms * per_sm[slot];
    if (blocks > cap) blocks = cap;
    return blocks < 1 ? 1 : (int)blocks;
}

}  // namespace hx
