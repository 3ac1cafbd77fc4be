// diag.cu -- device watchdog self-test.
//
// One CTA waits on an mbarrier that nothing ever arrives on, through the same
// bounded wait the tcgen05 kernels use, with a caller-chosen budget.  The wait
// gives up, sets the device error word and the kernel returns normally: the
// context stays usable and hexcuda_sync() reports HEXCUDA_ERR_TIMEOUT.  This
// is how failure detection is exercised without faulting or hanging a GPU.
#include "hx_internal.h"
#include "tc_common.cuh"

namespace hx {
namespace {

__global__ void watchdog_selftest_kernel(int *err_word, unsigned long long budget_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        abort_flag = 0;
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0)
        tc::mbar_wait(&bar, 0, &abort_flag, err_word, kErrWaitOther, budget_ns);
    __syncthreads();
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_selftest_watchdog(int dev, uint32_t budget_ms) {
    Dev *d = get_dev(dev);
    if (!d) return HEXCUDA_ERR_NODEV;
    if (budget_ms == 0 || budget_ms > 2000)
        return fail(HEXCUDA_ERR_ARG, "selftest_watchdog: budget %u ms (1..2000)", budget_ms);
    launch_begin(d);
    watchdog_selftest_kernel<<<1, 32, 0, d->stream>>>(d->err_word,
                                                      (unsigned long long)budget_ms * 1000000ull);
    return launch_end(d, "selftest_watchdog");
}
