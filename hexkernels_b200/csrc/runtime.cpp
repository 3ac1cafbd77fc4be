// runtime.cpp -- libhexcuda runtime: device set, streams, scratch pool,
// copies, errors and launch timing.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <vector>

#include "hx_internal.h"

namespace hx {

static std::vector<Dev> g_devs;
static bool g_inited = false;
static int g_last_err = HEXCUDA_OK;
static char g_last_msg[512] = "ok";
static bool g_timing = true;
static std::atomic<uint64_t> g_launches{0};
static std::atomic<unsigned> g_mech{0};
static float g_last_ms = -1.0f;
static bool g_last_ms_valid = false;

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
    va_end(ap);
    g_last_err = code;
    fprintf(stderr, "HEXCUDA_ERROR %d %s\n", code, g_last_msg);
    return code;
}

int check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return HEXCUDA_OK;
    return fail(e == cudaErrorMemoryAllocation ? HEXCUDA_ERR_OOM : HEXCUDA_ERR_CUDA,
                "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

static void release_all() {
    collective_release();
    for (auto &d : g_devs) {
        if (d.ordinal < 0) continue;
        cudaSetDevice(d.ordinal);
        cudaStreamSynchronize(d.stream);
        cudaStreamSynchronize(d.own_stream);
        for (int s = 0; s < kScratchSlots; s++)
            if (d.slot_ptr[s]) cudaFree(d.slot_ptr[s]);
        if (d.err_word) cudaFree(d.err_word);
        for (int k = 0; k < kPipeChunks; k++) {
            if (d.ev_in[k]) cudaEventDestroy(d.ev_in[k]);
            if (d.ev_done[k]) cudaEventDestroy(d.ev_done[k]);
        }
        if (d.s_in) cudaStreamDestroy(d.s_in);
        if (d.s_out) cudaStreamDestroy(d.s_out);
        if (d.ev0) cudaEventDestroy(d.ev0);
        if (d.ev1) cudaEventDestroy(d.ev1);
        if (d.own_stream) cudaStreamDestroy(d.own_stream);
    }
    g_devs.clear();
    g_inited = false;
}

static int init_list(const int *devs, int n) {
    if (g_inited) {
        bool same = (int)g_devs.size() == n;
        for (int i = 0; same && i < n; i++) same = g_devs[i].ordinal == devs[i];
        if (same) return HEXCUDA_OK;
        release_all();
    }
    int count = 0;
    if (int rc = check(cudaGetDeviceCount(&count), "cudaGetDeviceCount")) return rc;
    if (n <= 0) return fail(HEXCUDA_ERR_NODEV, "no device requested");
    g_devs.assign((size_t)n, Dev());
    for (int i = 0; i < n; i++) {
        Dev &d = g_devs[(size_t)i];
        if (devs[i] < 0 || devs[i] >= count) {
            release_all();
            return fail(HEXCUDA_ERR_NODEV, "device %d not present (%d visible)", devs[i], count);
        }
        cudaDeviceProp prop;
        int rc = check(cudaGetDeviceProperties(&prop, devs[i]), "cudaGetDeviceProperties");
        if (!rc && prop.major != 10) {
            release_all();
            return fail(HEXCUDA_ERR_NODEV,
                        "device %d is sm_%d%d; libhexcuda is built for sm_100a only",
                        devs[i], prop.major, prop.minor);
        }
        if (!rc) rc = check(cudaSetDevice(devs[i]), "cudaSetDevice");
        d.ordinal = devs[i];
        d.sms = prop.multiProcessorCount;
        if (!rc) rc = check(cudaStreamCreateWithFlags(&d.own_stream, cudaStreamNonBlocking),
                            "cudaStreamCreate");
        d.stream = d.own_stream;
        if (!rc) rc = check(cudaEventCreate(&d.ev0), "cudaEventCreate");
        if (!rc) rc = check(cudaEventCreate(&d.ev1), "cudaEventCreate");
        if (!rc) rc = check(cudaStreamCreateWithFlags(&d.s_in, cudaStreamNonBlocking),
                            "cudaStreamCreate(in)");
        if (!rc) rc = check(cudaStreamCreateWithFlags(&d.s_out, cudaStreamNonBlocking),
                            "cudaStreamCreate(out)");
        for (int k = 0; k < kPipeChunks && !rc; k++) {
            rc = check(cudaEventCreateWithFlags(&d.ev_in[k], cudaEventDisableTiming), "event");
            if (!rc) rc = check(cudaEventCreateWithFlags(&d.ev_done[k], cudaEventDisableTiming), "event");
        }
        if (!rc) rc = check(cudaMalloc(&d.err_word, 256), "cudaMalloc(err_word)");
        if (!rc) rc = check(cudaMemset(d.err_word, 0, 256), "cudaMemset(err_word)");
        if (rc) {
            release_all();
            return rc;
        }
    }
    g_inited = true;
    return HEXCUDA_OK;
}

bool ensure_init() {
    if (g_inited) return true;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
        fail(HEXCUDA_ERR_NODEV, "no CUDA device visible");
        return false;
    }
    // HEXCUDA_NGPUS limits how many devices the host entries shard over.
    const char *env = getenv("HEXCUDA_NGPUS");
    int n = env ? atoi(env) : 1;
    if (n <= 0 || n > count) n = count;
    std::vector<int> ids((size_t)n);
    for (int i = 0; i < n; i++) ids[(size_t)i] = i;
    return init_list(ids.data(), n) == HEXCUDA_OK;
}

int ndev() { return (int)g_devs.size(); }

Dev *get_dev(int slot) {
    if (!ensure_init()) return nullptr;
    if (slot < 0 || slot >= (int)g_devs.size()) {
        fail(HEXCUDA_ERR_NODEV, "device slot %d out of range (%d initialised)", slot,
             (int)g_devs.size());
        return nullptr;
    }
    Dev *d = &g_devs[(size_t)slot];
    if (check(cudaSetDevice(d->ordinal), "cudaSetDevice")) return nullptr;
    return d;
}

void *scratch(Dev *d, int slot, size_t bytes) {
    if (slot < 0 || slot >= kScratchSlots) {
        fail(HEXCUDA_ERR_ARG, "scratch slot %d out of range", slot);
        return nullptr;
    }
    if (bytes == 0) bytes = 256;
    if (d->slot_bytes[slot] >= bytes) return d->slot_ptr[slot];
    if (d->slot_ptr[slot]) {
        // the old buffer may still be read by queued work
        cudaStreamSynchronize(d->stream);
        cudaFree(d->slot_ptr[slot]);
        d->slot_ptr[slot] = nullptr;
        d->slot_bytes[slot] = 0;
    }
    if (slot == kSlotSplit) {
        // a new buffer: its flag region is zeroed again before first use
        d->split_zeroed = nullptr;
        d->split_zeroed_bytes = 0;
    }
    size_t want = (bytes + 4095) & ~(size_t)4095;
    void *p = nullptr;
    if (check(cudaMalloc(&p, want), "cudaMalloc(scratch)")) return nullptr;
    d->slot_ptr[slot] = p;
    d->slot_bytes[slot] = want;
    return p;
}

void note_mech(unsigned bits) { g_mech.fetch_or(bits); }

static bool g_scope = false;

void scope_begin() {
    g_scope = true;
    for (auto &d : g_devs) d.timed = d.ev0_recorded = false;
    g_last_ms_valid = false;
}

void scope_end() { g_scope = false; }

void launch_begin(Dev *d) {
    if (!g_scope) {
        // a lone device launch: the timing covers this launch only
        for (auto &o : g_devs) o.timed = o.ev0_recorded = false;
    }
    if (!g_timing || d->ev0_recorded) return;
    if (cudaEventRecord(d->ev0, d->stream) == cudaSuccess) d->ev0_recorded = true;
}

int launch_end(Dev *d, const char *name, int nlaunches) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        d->timed = d->ev0_recorded = false;
        return fail(HEXCUDA_ERR_CUDA, "launch %s: %s", name, cudaGetErrorString(e));
    }
    g_launches += (uint64_t)nlaunches;
    d->timed = d->ev0_recorded && cudaEventRecord(d->ev1, d->stream) == cudaSuccess;
    g_last_ms_valid = false;
    return HEXCUDA_OK;
}

}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_init(int ngpus) {
    int count = 0;
    if (int rc = check(cudaGetDeviceCount(&count), "cudaGetDeviceCount")) return rc;
    if (count <= 0) return fail(HEXCUDA_ERR_NODEV, "no CUDA device visible");
    if (ngpus <= 0 || ngpus > count) ngpus = count;
    std::vector<int> ids((size_t)ngpus);
    for (int i = 0; i < ngpus; i++) ids[(size_t)i] = i;
    return init_list(ids.data(), ngpus);
}

HX_EXPORT int hexcuda_init_devices(const int *devs, int n) {
    if (!devs || n <= 0) return fail(HEXCUDA_ERR_ARG, "empty device list");
    return init_list(devs, n);
}

HX_EXPORT void hexcuda_shutdown(void) { release_all(); }

HX_EXPORT int hexcuda_device_count(void) { return ensure_init() ? ndev() : 0; }

HX_EXPORT int hexcuda_device_ordinal(int slot) {
    Dev *d = get_dev(slot);
    return d ? d->ordinal : -1;
}

HX_EXPORT void *hexcuda_alloc(int dev, size_t bytes) {
    Dev *d = get_dev(dev);
    if (!d) return nullptr;
    void *p = nullptr;
    if (check(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc")) return nullptr;
    return p;
}

HX_EXPORT int hexcuda_free(int dev, void *ptr) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    return ptr ? check(cudaFree(ptr), "cudaFree") : HEXCUDA_OK;
}

HX_EXPORT void *hexcuda_host_alloc(size_t bytes) {
    void *p = nullptr;
    if (check(cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocPortable), "cudaHostAlloc"))
        return nullptr;
    return p;
}

HX_EXPORT int hexcuda_host_free(void *ptr) {
    return ptr ? check(cudaFreeHost(ptr), "cudaFreeHost") : HEXCUDA_OK;
}

HX_EXPORT int hexcuda_h2d(int dev, void *dst, const void *src, size_t bytes) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    if (!bytes) return HEXCUDA_OK;
    if (!dst || !src) return fail(HEXCUDA_ERR_ARG, "h2d: null pointer");
    return check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d->stream), "h2d");
}

HX_EXPORT int hexcuda_d2h(int dev, void *dst, const void *src, size_t bytes) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    if (!bytes) return HEXCUDA_OK;
    if (!dst || !src) return fail(HEXCUDA_ERR_ARG, "d2h: null pointer");
    return check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, d->stream), "d2h");
}

HX_EXPORT int hexcuda_memset(int dev, void *dst, int value, size_t bytes) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    if (!bytes) return HEXCUDA_OK;
    return check(cudaMemsetAsync(dst, value, bytes, d->stream), "memset");
}

static int sync_one(Dev *d) {
    if (int rc = check(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) return rc;
    int word = 0;
    if (int rc = check(cudaMemcpy(&word, d->err_word, sizeof(int), cudaMemcpyDeviceToHost),
                       "read watchdog word"))
        return rc;
    if (word) {
        cudaMemset(d->err_word, 0, sizeof(int));
        return fail(HEXCUDA_ERR_TIMEOUT,
                    "device %d: a bounded device-side wait expired (flags 0x%x); outputs of "
                    "the last launch are invalid",
                    d->ordinal, word);
    }
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_sync(int dev) {
    if (dev >= 0) {
        Dev *d = get_dev(dev);
        return d ? sync_one(d) : g_last_err;
    }
    if (!ensure_init()) return g_last_err;
    int rc = HEXCUDA_OK;
    for (int i = 0; i < ndev(); i++) {
        Dev *d = get_dev(i);
        int r = d ? sync_one(d) : g_last_err;
        if (r && !rc) rc = r;
    }
    return rc;
}

HX_EXPORT void *hexcuda_stream(int dev) {
    Dev *d = get_dev(dev);
    return d ? (void *)d->stream : nullptr;
}

HX_EXPORT int hexcuda_set_stream(int dev, void *stream) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    d->stream = (cudaStream_t)stream;
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_reset_stream(int dev) {
    Dev *d = get_dev(dev);
    if (!d) return g_last_err;
    d->stream = d->own_stream;
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_last_error(void) { return g_last_err; }
HX_EXPORT const char *hexcuda_last_error_string(void) { return g_last_msg; }

HX_EXPORT int hexcuda_set_timing(int on) {
    g_timing = on != 0;
    return HEXCUDA_OK;
}

HX_EXPORT float hexcuda_last_kernel_ms(void) {
    if (g_last_ms_valid) return g_last_ms;
    float best = -1.0f;
    for (auto &d : g_devs) {
        if (!d.timed) continue;
        cudaSetDevice(d.ordinal);
        if (cudaEventSynchronize(d.ev1) != cudaSuccess) continue;
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, d.ev0, d.ev1) == cudaSuccess && ms > best) best = ms;
    }
    g_last_ms = best;
    g_last_ms_valid = true;
    return best;
}

HX_EXPORT uint64_t hexcuda_launch_count(void) { return g_launches.load(); }

HX_EXPORT unsigned hexcuda_mechanisms(int reset) {
    return reset ? g_mech.exchange(0u) : g_mech.load();
}
