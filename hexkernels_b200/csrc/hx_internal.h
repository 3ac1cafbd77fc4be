// hx_internal.h -- shared internals of libhexcuda (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <vector>

#include "hexcuda.h"

#define HX_EXPORT extern "C" __attribute__((visibility("default")))

namespace hx {

constexpr int kScratchSlots = 26;
constexpr int kSlotReplica = 24;  // replicated output of the last host entry (collective.cpp)
constexpr int kSlotSplit = 25;    // GEMM tail split: arrival flags + partial accumulators (gemm.cu)
constexpr int kPipeChunks = 64;     // max chunks in flight per pipelined host call

// Per-device state.  `stream` is where every launcher enqueues work; it is the
// device's own non-blocking stream unless a caller installed another one.
struct Dev {
    int ordinal = -1;
    int sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    bool ev0_recorded = false;          // ev0 marks the start of the timed scope
    bool timed = false;                 // ev0/ev1 bracket the last launch(es)
    int *err_word = nullptr;            // device watchdog word (0 = ok)
    // copy streams and per-chunk events of the pipelined host entries
    cudaStream_t s_in = nullptr, s_out = nullptr;
    cudaEvent_t ev_in[kPipeChunks] = {}, ev_done[kPipeChunks] = {};
    void *slot_ptr[kScratchSlots] = {};
    size_t slot_bytes[kScratchSlots] = {};
    // the GEMM tail split's flag region: which buffer and how many bytes of
    // it have been zeroed (flags are only ever written with launch tickets)
    void *split_zeroed = nullptr;
    size_t split_zeroed_bytes = 0;
};

// Device slot -> state; records HEXCUDA_ERR_NODEV and returns null when the
// slot is invalid.  Makes the device current.
Dev *get_dev(int slot);
int ndev();
bool ensure_init();

// Error recording: prints "HEXCUDA_ERROR <code> <msg>" to stderr once per
// failure and returns `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int check(cudaError_t e, const char *what);

// Grow-only device buffer owned by libhexcuda, reused across calls.  Slots are
// assigned by the caller (each call site uses its own slot numbers).
void *scratch(Dev *d, int slot, size_t bytes);

// Bracket a kernel launch: records the timing events (when enabled) and, after
// the launch, checks cudaGetLastError and counts the launch.  Inside a scope
// (a host entry spanning several devices and launches) each device's event
// pair spans its first to its last launch.
void scope_begin();
void scope_end();
void launch_begin(Dev *d);
int launch_end(Dev *d, const char *name, int nlaunches = 1);

// Which kinds of kernel ran (hexcuda_mechanisms): the launchers of the
// tcgen05 / TMA kernels record their bits here at every launch.
enum : unsigned { kMechTcgen05 = 1u, kMechTma = 2u, kMechVec128 = 4u };
void note_mech(unsigned bits);

// Replicated outputs (collective.cpp): whether the caller asked for them, and
// the gather of the devices' row parts (douts[slot], null for an empty part)
// into every device's replica buffer, enqueued on each device's stream.
bool replicate_on();
int replicate_rows(const std::vector<void *> &douts, int64_t rows, size_t row_bytes);
void replica_clear();
void collective_release();

// Watchdog budget for device-side bounded waits, in nanoseconds of
// %globaltimer.  A wait that exceeds it sets the device error word.
constexpr unsigned long long kWaitBudgetNs = 4000000000ull;

// Error word codes set by kernels (bit flags, OR-ed).
enum : int {
    kErrWaitFull = 1,      // consumer wait on a filled-stage barrier expired
    kErrWaitEmpty = 2,     // producer wait on a free-stage barrier expired
    kErrWaitAccum = 4,     // accumulator hand-off wait expired
    kErrWaitOther = 8,
    kErrWaitPart = 16,     // GEMM tail split: wait for another CTA's partial expired
};

}  // namespace hx
