// host_entries.cpp -- host-pointer entry points (hexcuda_host_*): the calls
// the candidate_kernel shims make.  Rows are split into contiguous shards,
// one per initialised device.  Operators whose inputs and output are all
// row-sharded (row operators, GEMMs along M, attention along heads, the
// elementwise requant) pipeline each shard in chunks, copies in, kernels and
// copies out overlapping (run_pipelined); the others copy a shard in on that
// device's stream, compute, and only after every device finished without
// error copy back (run_sharded).  In both, an argument or launch error leaves
// the caller's output untouched.  Per-column / per-feature operands are
// replicated to every device.
#include <string.h>

#include <algorithm>
#include <functional>
#include <vector>

#include "hx_internal.h"

namespace hx {
namespace {

// staging slots of the device scratch pool used by the host entries
enum : int { kSlotIn0 = 8, kSlotIn1, kSlotIn2, kSlotIn3, kSlotIn4, kSlotIn5, kSlotOut };

struct Part {
    int slot;           // device slot
    Dev *d;
    int64_t r0, r1;     // shard of the row range
    void *dout;         // device output of this shard
};

template <typename T>
T *stage_in(Dev *d, int slot, const T *host, size_t count) {
    T *p = reinterpret_cast<T *>(scratch(d, slot, count * sizeof(T)));
    if (!p) return nullptr;
    if (count && check(cudaMemcpyAsync(p, host, count * sizeof(T), cudaMemcpyHostToDevice,
                                       d->stream),
                       "h2d"))
        return nullptr;
    return p;
}

// Runs `enqueue(part)` on every shard (it stages inputs, launches and sets
// part.dout), waits for all devices, then copies each shard's output rows
// [r0, r1) (out_row_bytes each) back into `host_out`.
// cm_cols > 0: the output is column-major [cm_cols][rows] with cm_esize-byte
// elements, each shard's device output column-major [cm_cols][r1 - r0].
int run_sharded(int64_t rows, void *host_out, size_t out_row_bytes,
                const std::function<int(Part &)> &enqueue, int64_t cm_cols = 0,
                size_t cm_esize = 0) {
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const int n = ndev();
    std::vector<Part> parts;
    for (int i = 0; i < n; i++) {
        int64_t r0 = rows * i / n, r1 = rows * (i + 1) / n;
        if (r1 > r0) parts.push_back(Part{i, nullptr, r0, r1, nullptr});
    }
    if (parts.empty()) return HEXCUDA_OK;
    scope_begin();
    int rc = HEXCUDA_OK;
    for (auto &p : parts) {
        p.d = get_dev(p.slot);
        if (!p.d) {
            rc = HEXCUDA_ERR_NODEV;
            break;
        }
        if ((rc = enqueue(p))) break;
    }
    if (!rc && replicate_on()) {
        // every device also receives the other devices' rows (row-major
        // outputs; a column-major store leaves no replica)
        if (cm_cols > 0) {
            replica_clear();
        } else {
            std::vector<void *> douts((size_t)n, nullptr);
            for (auto &p : parts) douts[(size_t)p.slot] = p.dout;
            rc = replicate_rows(douts, rows, out_row_bytes);
        }
    }
    for (auto &p : parts) {
        if (!p.d) continue;
        int r = hexcuda_sync(p.slot);
        if (r && !rc) rc = r;
    }
    scope_end();
    if (rc) return rc;
    for (auto &p : parts) {
        size_t bytes = (size_t)(p.r1 - p.r0) * out_row_bytes;
        if (!bytes) continue;
        cudaSetDevice(p.d->ordinal);
        if (cm_cols > 0) {
            const size_t w = (size_t)(p.r1 - p.r0) * cm_esize;
            if ((rc = check(cudaMemcpy2DAsync(reinterpret_cast<uint8_t *>(host_out) +
                                                  (size_t)p.r0 * cm_esize,
                                              (size_t)rows * cm_esize, p.dout, w, w,
                                              (size_t)cm_cols, cudaMemcpyDeviceToHost,
                                              p.d->stream),
                            "d2h (column-major)")))
                return rc;
            continue;
        }
        if ((rc = check(cudaMemcpyAsync(reinterpret_cast<uint8_t *>(host_out) + p.r0 * out_row_bytes,
                                        p.dout, bytes, cudaMemcpyDeviceToHost, p.d->stream),
                        "d2h")))
            return rc;
    }
    for (auto &p : parts)
        if (int r = hexcuda_sync(p.slot)) return r;
    return HEXCUDA_OK;
}

// One row-sharded input of a pipelined call: `host` holds the call's rows of
// `row_bytes` bytes each; a device stages its shard in scratch slot `slot`.
struct RowIn {
    const void *host;
    size_t row_bytes;
    int slot;
};
constexpr int kMaxRowIns = 4;

// launch(part, device inputs (one per RowIn, at the chunk's first row),
//        device output at the chunk's first row, rows in the chunk)
using ChunkLaunch = std::function<int(Part &, const uint8_t *const *, void *, int64_t)>;

// Pipelined variant of run_sharded for operators whose inputs and output are
// all row-sharded apart from replicated operands (the row operators, GEMMs
// cut along M, attention cut along heads).  Each device's shard is cut into
// up to kPipeChunks chunks of about `chunk_bytes` (counted on the larger of
// a row's input and output bytes); chunk k is copied in on the device's input
// stream, computed on its launch stream once its copies have landed (event),
// and copied out on its output stream once its kernels have finished
// (event).  With pinned host memory the two copy directions and the kernels
// of different chunks overlap.  Chunks hold a multiple of 16 rows, so a
// chunk starts 16-byte aligned whenever a row's bytes are a multiple of 16
// (what the TMA operands need).  All copies in and launches are enqueued
// before any copy out, so an argument or launch error still leaves the
// caller's output untouched.
int run_pipelined(int64_t rows, std::initializer_list<RowIn> in_list, void *host_out,
                  size_t out_row_bytes, int64_t chunk_bytes,
                  const std::function<int(Part &)> &stage_replicated, const ChunkLaunch &launch) {
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const std::vector<RowIn> ins(in_list);
    if (ins.empty() || ins.size() > (size_t)kMaxRowIns)
        return fail(HEXCUDA_ERR_ARG, "pipelined call with %zu inputs", ins.size());
    size_t row_bytes = out_row_bytes, in_row = 0;
    for (const RowIn &in : ins) in_row += in.row_bytes;
    row_bytes = std::max(row_bytes, in_row);
    const int n = ndev();
    std::vector<Part> parts;
    for (int i = 0; i < n; i++) {
        int64_t r0 = rows * i / n, r1 = rows * (i + 1) / n;
        if (r1 > r0) parts.push_back(Part{i, nullptr, r0, r1, nullptr});
    }
    if (parts.empty()) return HEXCUDA_OK;
    struct Plan {
        uint8_t *din[kMaxRowIns];
        uint8_t *dout;
        int64_t chunk, nchunks;
    };
    std::vector<Plan> plans(parts.size());
    scope_begin();
    int rc = HEXCUDA_OK;
    for (size_t pi = 0; pi < parts.size() && !rc; pi++) {
        Part &p = parts[pi];
        Plan &pl = plans[pi];
        p.d = get_dev(p.slot);
        if (!p.d) {
            rc = HEXCUDA_ERR_NODEV;
            break;
        }
        const int64_t nr = p.r1 - p.r0;
        for (size_t i = 0; i < ins.size() && !rc; i++) {
            pl.din[i] = reinterpret_cast<uint8_t *>(
                scratch(p.d, ins[i].slot, (size_t)nr * ins[i].row_bytes));
            if (!pl.din[i]) rc = hexcuda_last_error();
        }
        pl.dout = reinterpret_cast<uint8_t *>(scratch(p.d, kSlotOut, (size_t)nr * out_row_bytes));
        if (!rc && !pl.dout) rc = hexcuda_last_error();
        if (rc) break;
        p.dout = pl.dout;
        int64_t chunk = std::max<int64_t>(1, chunk_bytes / (int64_t)std::max<size_t>(row_bytes, 1));
        chunk = std::max(chunk, (nr + kPipeChunks - 1) / kPipeChunks);
        chunk = (chunk + 15) / 16 * 16;
        pl.chunk = std::min(chunk, nr);
        pl.nchunks = (nr + pl.chunk - 1) / pl.chunk;
        // replicated operands go first on the input stream, so every chunk's
        // input event also covers them
        cudaStream_t launch_stream = p.d->stream;
        p.d->stream = p.d->s_in;
        rc = stage_replicated(p);
        p.d->stream = launch_stream;
        const uint8_t *dchunk[kMaxRowIns] = {};
        for (int64_t k = 0; k < pl.nchunks && !rc; k++) {
            const int64_t c0 = k * pl.chunk, cn = std::min(pl.chunk, nr - c0);
            for (size_t i = 0; i < ins.size() && !rc; i++) {
                const size_t rb = ins[i].row_bytes;
                dchunk[i] = pl.din[i] + c0 * rb;
                if (rb)
                    rc = check(cudaMemcpyAsync(pl.din[i] + c0 * rb,
                                               reinterpret_cast<const uint8_t *>(ins[i].host) +
                                                   (p.r0 + c0) * rb,
                                               (size_t)cn * rb, cudaMemcpyHostToDevice, p.d->s_in),
                               "h2d");
            }
            if (!rc) rc = check(cudaEventRecord(p.d->ev_in[k], p.d->s_in), "event");
            if (!rc) rc = check(cudaStreamWaitEvent(p.d->stream, p.d->ev_in[k], 0), "wait event");
            if (!rc) rc = launch(p, dchunk, pl.dout + c0 * out_row_bytes, cn);
            if (!rc) rc = check(cudaEventRecord(p.d->ev_done[k], p.d->stream), "event");
        }
    }
    if (!rc && replicate_on()) {
        std::vector<void *> douts((size_t)n, nullptr);
        for (size_t pi = 0; pi < parts.size(); pi++) douts[(size_t)parts[pi].slot] = plans[pi].dout;
        rc = replicate_rows(douts, rows, out_row_bytes);
    }
    if (!rc) {
        for (size_t pi = 0; pi < parts.size() && !rc; pi++) {
            Part &p = parts[pi];
            Plan &pl = plans[pi];
            cudaSetDevice(p.d->ordinal);
            const int64_t nr = p.r1 - p.r0;
            for (int64_t k = 0; k < pl.nchunks && !rc; k++) {
                const int64_t c0 = k * pl.chunk, cn = std::min(pl.chunk, nr - c0);
                rc = check(cudaStreamWaitEvent(p.d->s_out, p.d->ev_done[k], 0), "wait event");
                if (!rc)
                    rc = check(cudaMemcpyAsync(reinterpret_cast<uint8_t *>(host_out) +
                                                   (p.r0 + c0) * out_row_bytes,
                                               pl.dout + c0 * out_row_bytes,
                                               (size_t)cn * out_row_bytes, cudaMemcpyDeviceToHost,
                                               p.d->s_out),
                               "d2h");
            }
        }
    }
    for (auto &p : parts) {
        if (!p.d) continue;
        cudaSetDevice(p.d->ordinal);
        int r = check(cudaStreamSynchronize(p.d->s_in), "sync in");
        if (!r) r = check(cudaStreamSynchronize(p.d->s_out), "sync out");
        if (!r) r = hexcuda_sync(p.slot);
        if (r && !rc) rc = r;
    }
    scope_end();
    return rc;
}

// Chunk size of the pipelined entries: 32 MiB for the row operators, 16 MiB
// for GEMMs along M and attention along heads.  Measured through the host
// entries with pinned buffers on one B200 (two runs each): the fp32
// softmax + layernorm pair over 65536 x 4096 moved 91.7 GB/s with 32 MiB
// chunks and 86.1 GB/s with 8 MiB chunks (smaller copies cost more per byte
// than their shorter fill and drain save); the benchmark GEMMs and attention
// ran 1-7 % slower with 8 MiB chunks than with 16 MiB.
// HEXCUDA_PIPE_CHUNK_MB overrides both (a tuning knob).
int64_t pipe_chunk_bytes(int64_t dflt) {
    static int64_t env = -1;
    if (env < 0) {
        const char *e = getenv("HEXCUDA_PIPE_CHUNK_MB");
        env = (e && atoi(e) > 0) ? (int64_t)atoi(e) << 20 : 0;
    }
    return env > 0 ? env : dflt;
}
constexpr int64_t kRowChunkBytes = 32ll << 20;
constexpr int64_t kGemmChunkBytes = 16ll << 20;

// The row operators: one row-sharded input.
int run_rows_pipelined(int64_t rows, const void *host_in, size_t in_row_bytes, void *host_out,
                       size_t out_row_bytes, const std::function<int(Part &)> &stage_replicated,
                       const std::function<int(Part &, const void *, void *, int64_t)> &launch) {
    return run_pipelined(rows, {RowIn{host_in, in_row_bytes, kSlotIn0}}, host_out, out_row_bytes,
                         pipe_chunk_bytes(kRowChunkBytes), stage_replicated,
                         [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
                             return launch(p, din[0], dout, nr);
                         });
}

// Number of per-device slots for a call's replicated operands.  The library
// is initialised first (a host entry may be the process's first call), so
// this is the number of devices the call shards over; 0 when no device is
// visible, and the call then fails in run_sharded / run_pipelined before any
// slot is used.
inline size_t dev_count() { return ensure_init() ? (size_t)ndev() : 0; }

inline int null_check(const char *name, std::initializer_list<const void *> ptrs) {
    for (const void *p : ptrs)
        if (!p) return fail(HEXCUDA_ERR_ARG, "%s: null pointer", name);
    return HEXCUDA_OK;
}

}  // namespace
}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_host_softmax_f32(const float *x, float *out, int R, int C) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_softmax_f32: R=%d C=%d", R, C);
    if (int rc = null_check("host_softmax_f32", {x, out})) return rc;
    const size_t rb = sizeof(float) * (size_t)C;
    return run_rows_pipelined(
        R, x, rb, out, rb, [](Part &) { return HEXCUDA_OK; },
        [&](Part &p, const void *din, void *dout, int64_t nr) {
            return hexcuda_softmax_f32(p.slot, (const float *)din, (float *)dout, (int)nr, C);
        });
}

HX_EXPORT int hexcuda_host_softmax_f16(const uint16_t *x, uint16_t *out, int R, int C) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_softmax_f16: R=%d C=%d", R, C);
    if (int rc = null_check("host_softmax_f16", {x, out})) return rc;
    const size_t rb = 2 * (size_t)C;
    return run_rows_pipelined(
        R, x, rb, out, rb, [](Part &) { return HEXCUDA_OK; },
        [&](Part &p, const void *din, void *dout, int64_t nr) {
            return hexcuda_softmax_f16(p.slot, (const uint16_t *)din, (uint16_t *)dout, (int)nr, C);
        });
}

HX_EXPORT int hexcuda_host_layernorm_f32(const float *x, const float *gamma, const float *beta,
                                         float *out, int R, int C, float eps) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_layernorm_f32: R=%d C=%d", R, C);
    if (int rc = null_check("host_layernorm_f32", {x, gamma, beta, out})) return rc;
    const size_t rb = sizeof(float) * (size_t)C;
    std::vector<const float *> dg(dev_count()), db(dev_count());
    return run_rows_pipelined(
        R, x, rb, out, rb,
        [&](Part &p) {
            dg[p.slot] = stage_in(p.d, kSlotIn1, gamma, (size_t)C);
            db[p.slot] = stage_in(p.d, kSlotIn2, beta, (size_t)C);
            return (dg[p.slot] && db[p.slot]) ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const void *din, void *dout, int64_t nr) {
            return hexcuda_layernorm_f32(p.slot, (const float *)din, dg[p.slot], db[p.slot],
                                         (float *)dout, (int)nr, C, eps);
        });
}

HX_EXPORT int hexcuda_host_layernorm_f16(const uint16_t *x, const uint16_t *gamma,
                                         const uint16_t *beta, uint16_t *out, int R, int C,
                                         float eps) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_layernorm_f16: R=%d C=%d", R, C);
    if (int rc = null_check("host_layernorm_f16", {x, gamma, beta, out})) return rc;
    return run_sharded(R, out, 2 * (size_t)C, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const uint16_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const uint16_t *dg = stage_in(p.d, kSlotIn1, gamma, (size_t)C);
        const uint16_t *db = stage_in(p.d, kSlotIn2, beta, (size_t)C);
        uint16_t *dout = reinterpret_cast<uint16_t *>(scratch(p.d, kSlotOut, 2 * nr * C));
        if (!dx || !dg || !db || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_layernorm_f16(p.slot, dx, dg, db, dout, (int)nr, C, eps);
    });
}

HX_EXPORT int hexcuda_host_rmsnorm_gain_f16(const uint16_t *x, const uint16_t *gain, uint16_t *out,
                                            int R, int C, float eps) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_rmsnorm_gain_f16: R=%d C=%d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_rmsnorm_gain_f16", {x, gain, out})) return rc;
    return run_sharded(R, out, 2 * (size_t)C, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const uint16_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const uint16_t *dg = stage_in(p.d, kSlotIn1, gain + p.r0, (size_t)nr);
        uint16_t *dout = reinterpret_cast<uint16_t *>(scratch(p.d, kSlotOut, 2 * nr * C));
        if (!dx || !dg || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_rmsnorm_gain_f16(p.slot, dx, dg, dout, (int)nr, C, eps);
    });
}

HX_EXPORT int hexcuda_host_rmsnorm_f16(const uint16_t *x, const uint16_t *gamma, uint16_t *out,
                                       int R, int C, float eps) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_rmsnorm_f16: R=%d C=%d", R, C);
    if (int rc = null_check("host_rmsnorm_f16", {x, gamma, out})) return rc;
    return run_sharded(R, out, 2 * (size_t)C, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const uint16_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const uint16_t *dg = stage_in(p.d, kSlotIn1, gamma, (size_t)C);
        uint16_t *dout = reinterpret_cast<uint16_t *>(scratch(p.d, kSlotOut, 2 * nr * C));
        if (!dx || !dg || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_rmsnorm_f16(p.slot, dx, dg, dout, (int)nr, C, eps);
    });
}

HX_EXPORT int hexcuda_host_rowreduce_f32(const float *x, float *out, int R, int C, int op) {
    if (R < 0 || C <= 0) return fail(HEXCUDA_ERR_ARG, "host_rowreduce_f32: R=%d C=%d", R, C);
    if (int rc = null_check("host_rowreduce_f32", {x, out})) return rc;
    return run_rows_pipelined(
        R, x, sizeof(float) * (size_t)C, out, sizeof(float), [](Part &) { return HEXCUDA_OK; },
        [&](Part &p, const void *din, void *dout, int64_t nr) {
            return hexcuda_rowreduce_f32(p.slot, (const float *)din, (float *)dout, (int)nr, C, op);
        });
}

HX_EXPORT int hexcuda_host_requant_per_channel(const int32_t *a, int8_t *out, int R, int C,
                                               const int32_t *mult, const int *shift, int8_t zp) {
    if (R < 0 || C < 0) return fail(HEXCUDA_ERR_ARG, "host_requant_per_channel: R=%d C=%d", R, C);
    if (R == 0 || C == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_requant_per_channel", {a, out, mult, shift})) return rc;
    return run_sharded(R, out, (size_t)C, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const int32_t *da = stage_in(p.d, kSlotIn0, a + p.r0 * C, (size_t)(nr * C));
        const int32_t *dm = stage_in(p.d, kSlotIn1, mult + p.r0, (size_t)nr);
        const int *ds = stage_in(p.d, kSlotIn2, shift + p.r0, (size_t)nr);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * C)));
        if (!da || !dm || !ds || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_requant_per_channel(p.slot, da, dout, (int)nr, C, dm, ds, zp);
    });
}

HX_EXPORT int hexcuda_host_requantize_i32_u8(const int32_t *a, uint8_t *out, int64_t n,
                                             int32_t mult, int shift, uint8_t zp) {
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "host_requantize_i32_u8: n=%lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_requantize_i32_u8", {a, out})) return rc;
    // rows of 4096 elements (the last one ragged) keep every chunk 16-byte aligned
    const int64_t rowlen = 4096, full = n / rowlen, tail = n - full * rowlen;
    int rc = HEXCUDA_OK;
    if (full > 0)
        rc = run_rows_pipelined(
            full, a, 4 * rowlen, out, rowlen, [](Part &) { return HEXCUDA_OK; },
            [&](Part &p, const void *din, void *dout, int64_t nr) {
                return hexcuda_requantize_i32_u8(p.slot, (const int32_t *)din, (uint8_t *)dout,
                                                 nr * rowlen, mult, shift, zp);
            });
    if (rc || tail == 0) return rc;
    return run_sharded(1, out + full * rowlen, (size_t)tail, [&](Part &p) {
        const int32_t *da = stage_in(p.d, kSlotIn0, a + full * rowlen, (size_t)tail);
        uint8_t *dout = reinterpret_cast<uint8_t *>(scratch(p.d, kSlotOut, (size_t)tail));
        if (!da || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_requantize_i32_u8(p.slot, da, dout, tail, mult, shift, zp);
    });
}

HX_EXPORT int hexcuda_host_gemm_i8_requant(const int8_t *A, const int8_t *B, int8_t *out, int M,
                                           int N, int K, int32_t mult, int shift, int8_t zp) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_requant: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i8_requant", {A, B, out})) return rc;
    return run_sharded(M, out, (size_t)N, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * N)));
        if (!dA || !dB || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_i8_requant(p.slot, dA, dB, dout, (int)nr, N, K, mult, shift, zp);
    });
}

HX_EXPORT int hexcuda_host_gemm_i8_bias_requant(const int8_t *A, const int8_t *B,
                                                const int32_t *bias, int8_t *out, int M, int N,
                                                int K, int32_t mult, int shift, int8_t zp) {
    if (M < 0 || N < 0 || K < 0)
        return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_bias_requant: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i8_bias_requant", {A, B, bias, out})) return rc;
    return run_sharded(M, out, (size_t)N, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        const int32_t *dbias = stage_in(p.d, kSlotIn2, bias, (size_t)N);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * N)));
        if (!dA || !dB || !dbias || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_i8_bias_requant(p.slot, dA, dB, dbias, dout, (int)nr, N, K, mult,
                                            shift, zp);
    });
}

HX_EXPORT int hexcuda_host_gemm_i8_zp(const int8_t *A, const int8_t *B, int8_t *out, int M, int N,
                                      int K, int32_t zpA, int32_t scale_mult, int scale_shift) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_zp: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i8_zp", {A, B, out})) return rc;
    return run_sharded(M, out, (size_t)N, [&](Part &p) {
        int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * N)));
        if (!dA || !dB || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_i8_zp(p.slot, dA, dB, dout, (int)nr, N, K, zpA, scale_mult,
                                  scale_shift);
    });
}

HX_EXPORT int hexcuda_host_gemm_u8s8_pc(const uint8_t *A, const int8_t *B, const int32_t *bias,
                                        uint8_t *out, int M, int N, int K, int32_t zpA,
                                        const int32_t *mult, const int *shift, uint8_t zp_out) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_u8s8_pc: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_u8s8_pc", {A, B, bias, out, mult, shift})) return rc;
    struct Rep {
        const int8_t *B;
        const int32_t *bias, *mult;
        const int *shift;
    };
    std::vector<Rep> rep(dev_count());
    return run_pipelined(
        M, {RowIn{A, (size_t)K, kSlotIn0}}, out, (size_t)N,
        pipe_chunk_bytes(kGemmChunkBytes),
        [&](Part &p) {
            Rep &r = rep[(size_t)p.slot];
            r.B = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
            r.bias = stage_in(p.d, kSlotIn2, bias, (size_t)N);
            r.mult = stage_in(p.d, kSlotIn3, mult, (size_t)N);
            r.shift = stage_in(p.d, kSlotIn4, shift, (size_t)N);
            return (r.B && r.bias && r.mult && r.shift) ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            const Rep &r = rep[(size_t)p.slot];
            return hexcuda_gemm_u8s8_pc(p.slot, din[0], r.B, r.bias, (uint8_t *)dout, (int)nr, N,
                                        K, zpA, r.mult, r.shift, zp_out);
        });
}

HX_EXPORT int hexcuda_host_requant_ew(const void *a, int a_i8, const void *b, int b_kind,
                                      void *out, int64_t n, int pre, int64_t pre_c, int32_t mult,
                                      int shift, int zp, int sign_of_a, int lo1, int hi1, int lo2,
                                      int hi2, const int8_t *lut) {
    if (n < 0 || b_kind < 0 || b_kind > 2) return fail(HEXCUDA_ERR_ARG, "host_requant_ew: bad size");
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_requant_ew", {a, out, b_kind ? b : a})) return rc;
    const size_t ea = a_i8 ? 1 : 4, eb = b_kind == 2 ? 1 : 4;
    std::vector<const int8_t *> dl(dev_count());
    // one element per row; chunks of a multiple of 16 elements keep every
    // operand's chunk 16-byte aligned
    return run_pipelined(
        n, {RowIn{a, ea, kSlotIn0}, RowIn{b, b_kind ? eb : 0, kSlotIn1}}, out, 1,
        pipe_chunk_bytes(kRowChunkBytes),
        [&](Part &p) {
            dl[(size_t)p.slot] = lut ? stage_in(p.d, kSlotIn2, lut, 256) : nullptr;
            return (!lut || dl[(size_t)p.slot]) ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            return hexcuda_requant_ew(p.slot, din[0], a_i8, b_kind ? din[1] : nullptr, b_kind,
                                      dout, nr, pre, pre_c, mult, shift, zp, sign_of_a, lo1, hi1,
                                      lo2, hi2, dl[(size_t)p.slot]);
        });
}

HX_EXPORT int hexcuda_host_epilogue_bias_i32(const int32_t *acc, const int32_t *bias,
                                             int32_t *out, int R, int C) {
    if (R < 0 || C < 0) return fail(HEXCUDA_ERR_ARG, "host_epilogue_bias_i32: bad shape");
    if (R == 0 || C == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_epilogue_bias_i32", {acc, bias, out})) return rc;
    return run_sharded(R, out, (size_t)C * 4, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int32_t *dacc = stage_in(p.d, kSlotIn0, acc + p.r0 * C, (size_t)(nr * C));
        const int32_t *dbias = stage_in(p.d, kSlotIn1, bias, (size_t)C);
        int32_t *dout = reinterpret_cast<int32_t *>(scratch(p.d, kSlotOut, (size_t)(nr * C) * 4));
        if (!dacc || !dbias || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_epilogue_bias_i32(p.slot, dacc, dbias, dout, (int)nr, C);
    });
}

HX_EXPORT int hexcuda_host_relu_i8(const int8_t *x, int8_t *out, int64_t n) {
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "host_relu_i8: n=%lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_relu_i8", {x, out})) return rc;
    return run_sharded(n, out, 1, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dx = stage_in(p.d, kSlotIn0, x + p.r0, (size_t)nr);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)nr));
        if (!dx || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_relu_i8(p.slot, dx, dout, nr);
    });
}

HX_EXPORT int hexcuda_host_gemm_hmx_ex(const uint8_t *A, const int8_t *B, int b_transposed,
                                       const int32_t *bias, const void *res, int res_kind,
                                       const void *lut, void *out, int store, int act,
                                       int col_major, int M, int N, int K, int32_t zpA) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_hmx: bad shape");
    if (store < HEXCUDA_HMX_STORE_I32 || store > HEXCUDA_HMX_STORE_ACC_I32 ||
        res_kind < HEXCUDA_HMX_RES_NONE || res_kind > HEXCUDA_HMX_RES_I8)
        return fail(HEXCUDA_ERR_ARG, "host_gemm_hmx: store %d / residual %d", store, res_kind);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    const bool has_lut = store == HEXCUDA_HMX_STORE_LUT_I32 || store == HEXCUDA_HMX_STORE_LUT_I8;
    if (int rc = null_check("host_gemm_hmx", {A, B, out, res_kind ? res : (const void *)A,
                                              has_lut ? lut : (const void *)A}))
        return rc;
    const size_t osize = (store == HEXCUDA_HMX_STORE_I32 || store == HEXCUDA_HMX_STORE_LUT_I32 ||
                          store == HEXCUDA_HMX_STORE_ACC_I32) ? 4
                         : store == HEXCUDA_HMX_STORE_U16_FIELD ? 2 : 1;
    const size_t rsize = res_kind == HEXCUDA_HMX_RES_I32 ? 4 : 1;
    const size_t lsize = store == HEXCUDA_HMX_STORE_LUT_I32 ? 4 : 1;
    if (!col_major) {
        struct Rep {
            const int8_t *B;
            const int32_t *bias;
            const uint8_t *lut;
        };
        std::vector<Rep> rep(dev_count());
        return run_pipelined(
            M,
            {RowIn{A, (size_t)K, kSlotIn0},
             RowIn{res, res_kind ? (size_t)N * rsize : 0, kSlotIn3}},
            out, (size_t)N * osize, pipe_chunk_bytes(kGemmChunkBytes),
            [&](Part &p) {
                Rep &r = rep[(size_t)p.slot];
                r.B = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
                r.bias = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
                r.lut = has_lut ? stage_in(p.d, kSlotIn4, reinterpret_cast<const uint8_t *>(lut),
                                           256 * lsize)
                                : nullptr;
                return (r.B && (!bias || r.bias) && (!has_lut || r.lut)) ? HEXCUDA_OK
                                                                         : hexcuda_last_error();
            },
            [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
                const Rep &r = rep[(size_t)p.slot];
                return hexcuda_gemm_hmx_ex(p.slot, din[0], r.B, b_transposed, r.bias,
                                           res_kind ? din[1] : nullptr, res_kind, r.lut, dout,
                                           store, act, 0, (int)nr, N, K, zpA);
            });
    }
    return run_sharded(
        M, out, (size_t)N * osize,
        [&](Part &p) {
            int64_t nr = p.r1 - p.r0;
            const uint8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
            const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
            const int32_t *dbias = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
            const uint8_t *dres =
                res_kind ? stage_in(p.d, kSlotIn3,
                                    reinterpret_cast<const uint8_t *>(res) + p.r0 * N * rsize,
                                    (size_t)(nr * N) * rsize)
                         : nullptr;
            const uint8_t *dlut =
                has_lut ? stage_in(p.d, kSlotIn4, reinterpret_cast<const uint8_t *>(lut), 256 * lsize)
                        : nullptr;
            void *dout = scratch(p.d, kSlotOut, (size_t)(nr * N) * osize);
            if (!dA || !dB || (bias && !dbias) || (res_kind && !dres) || (has_lut && !dlut) || !dout)
                return hexcuda_last_error();
            p.dout = dout;
            return hexcuda_gemm_hmx_ex(p.slot, dA, dB, b_transposed, dbias, dres, res_kind, dlut,
                                       dout, store, act, col_major, (int)nr, N, K, zpA);
        },
        col_major ? N : 0, osize);
}

HX_EXPORT int hexcuda_host_gemm_hmx(const uint8_t *A, const int8_t *B, int b_transposed,
                                    const int32_t *bias, void *out, int out_kind, int M, int N,
                                    int K, int32_t zpA) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_hmx: bad shape");
    if (out_kind < HEXCUDA_HMX_OUT_I32 || out_kind > HEXCUDA_HMX_OUT_U8_BIAS_RELU)
        return fail(HEXCUDA_ERR_ARG, "host_gemm_hmx: out_kind %d", out_kind);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    const bool has_bias = out_kind == HEXCUDA_HMX_OUT_U8_BIAS_RELU;
    if (int rc = null_check("host_gemm_hmx", {A, B, out, has_bias ? bias : (const void *)A}))
        return rc;
    const size_t osize = out_kind == HEXCUDA_HMX_OUT_I32 ? 4 : 1;
    std::vector<const int8_t *> dB(dev_count());
    std::vector<const int32_t *> dbias(dev_count());
    return run_pipelined(
        M, {RowIn{A, (size_t)K, kSlotIn0}}, out, (size_t)N * osize,
        pipe_chunk_bytes(kGemmChunkBytes),
        [&](Part &p) {
            const size_t s = (size_t)p.slot;
            dB[s] = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
            dbias[s] = has_bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
            return (dB[s] && (!has_bias || dbias[s])) ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            const size_t s = (size_t)p.slot;
            return hexcuda_gemm_hmx(p.slot, din[0], dB[s], b_transposed, dbias[s], dout, out_kind,
                                    (int)nr, N, K, zpA);
        });
}

HX_EXPORT int hexcuda_host_attn_qkt_av_hmx(const uint8_t *Q, const int8_t *K, const int8_t *V,
                                           int32_t *out, int SQ, int SK, int D) {
    if (SQ < 0 || SK < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "host_attn_qkt_av_hmx: bad shape");
    if (SQ == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_attn_qkt_av_hmx", {Q, K, V, out})) return rc;
    return run_sharded(SQ, out, (size_t)D * 4, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *dQ = stage_in(p.d, kSlotIn0, Q + p.r0 * D, (size_t)(nr * D));
        const int8_t *dK = stage_in(p.d, kSlotIn1, K, (size_t)SK * D);
        const int8_t *dV = stage_in(p.d, kSlotIn2, V, (size_t)SK * D);
        int32_t *dout = reinterpret_cast<int32_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D) * 4));
        if (!dQ || !dK || !dV || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_attn_qkt_av_hmx(p.slot, dQ, dK, dV, dout, (int)nr, SK, D);
    });
}

HX_EXPORT int hexcuda_host_attn_lut_i8(int mode, const void *Q, const int8_t *K, const int8_t *V,
                                       const uint8_t *exp_lut, const int8_t *cos_lut,
                                       const int8_t *sin_lut, int rot_shift, void *out, int HQ,
                                       int HKV, int S, int D, int32_t scale_mult, int scale_shift,
                                       int32_t av_mult, int av_shift) {
    if (HQ < 1 || HKV < 1 || HQ % HKV != 0 || S < 0 || D < 0)
        return fail(HEXCUDA_ERR_ARG, "host_attn_lut_i8: heads %d/%d S %d D %d", HQ, HKV, S, D);
    if (S == 0 || D == 0) return HEXCUDA_OK;
    const bool rope = mode == HEXCUDA_ATTN_LUT_HMX_ROPE;
    const void *cl = rope ? (const void *)cos_lut : (const void *)exp_lut;
    const void *sl = rope ? (const void *)sin_lut : (const void *)exp_lut;
    if (int rc = null_check("host_attn_lut_i8", {Q, K, V, exp_lut, out, cl, sl}))
        return rc;
    const size_t osize = mode == HEXCUDA_ATTN_LUT_REQUANT ? 1 : 2;
    const size_t hsd = (size_t)S * D;
    // one device: the blocks are small (one CTA per query head)
    return run_sharded(1, out, (size_t)HQ * hsd * osize, [&](Part &p) {
        const uint8_t *dQ = stage_in(p.d, kSlotIn0, reinterpret_cast<const uint8_t *>(Q), HQ * hsd);
        const int8_t *dK = stage_in(p.d, kSlotIn1, K, HKV * hsd);
        const int8_t *dV = stage_in(p.d, kSlotIn2, V, HKV * hsd);
        const uint8_t *dl = stage_in(p.d, kSlotIn3, exp_lut, 256);
        const size_t tab = (size_t)S * (D / 2);
        const int8_t *dc = rope ? stage_in(p.d, kSlotIn4, cos_lut, tab) : nullptr;
        const int8_t *ds = rope ? stage_in(p.d, kSlotIn5, sin_lut, tab) : nullptr;
        void *dout = scratch(p.d, kSlotOut, HQ * hsd * osize);
        if (!dQ || !dK || !dV || !dl || (rope && (!dc || !ds)) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_attn_lut_i8(p.slot, mode, dQ, dK, dV, dl, dc, ds, rot_shift, dout, HQ, HKV, S, D,
                                   scale_mult, scale_shift, av_mult, av_shift);
    });
}

HX_EXPORT int hexcuda_host_attn_lut_i8_window(const int8_t *Q, const int8_t *K, const int8_t *V,
                                              const uint8_t *exp_lut, int8_t *out, int H, int S,
                                              int D, int window, int32_t scale_mult,
                                              int scale_shift, int32_t av_mult, int av_shift) {
    if (H < 1 || S < 0 || D < 0 || window < 0)
        return fail(HEXCUDA_ERR_ARG, "host_attn_lut_i8_window: H %d S %d D %d window %d", H, S, D,
                    window);
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_attn_lut_i8_window", {Q, K, V, exp_lut, out})) return rc;
    const size_t n = (size_t)H * S * D;
    return run_sharded(1, out, n, [&](Part &p) {
        const int8_t *dQ = stage_in(p.d, kSlotIn0, Q, n);
        const int8_t *dK = stage_in(p.d, kSlotIn1, K, n);
        const int8_t *dV = stage_in(p.d, kSlotIn2, V, n);
        const uint8_t *dl = stage_in(p.d, kSlotIn3, exp_lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, n));
        if (!dQ || !dK || !dV || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_attn_lut_i8_window(p.slot, dQ, dK, dV, dl, dout, H, S, D, window, scale_mult,
                                          scale_shift, av_mult, av_shift);
    });
}

HX_EXPORT int hexcuda_host_decoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                            const int8_t *act_lut, const int8_t *W2,
                                            const int32_t *b2, const uint8_t *exp_lut, int8_t *out,
                                            int S, int D, int Dff) {
    if (S < 0 || D < 0 || Dff < 0) return fail(HEXCUDA_ERR_ARG, "host_decoder_block_i8: bad shape");
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_decoder_block_i8", {X, W1, b1, act_lut, W2, b2, exp_lut, out}))
        return rc;
    return run_sharded(1, out, (size_t)S * D, [&](Part &p) {
        const uint8_t *dX = stage_in(p.d, kSlotIn0, X, (size_t)S * D);
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)D * Dff);
        const int8_t *dW2 = stage_in(p.d, kSlotIn2, W2, (size_t)Dff * D);
        const int32_t *db1 = stage_in(p.d, kSlotIn3, b1, (size_t)Dff);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        // the two 256-entry tables share one slot
        uint8_t *tabs = reinterpret_cast<uint8_t *>(scratch(p.d, kSlotIn5, 512));
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)S * D));
        if (!dX || !dW1 || !dW2 || !db1 || !db2 || !tabs || !dout) return hexcuda_last_error();
        if (int rc = check(cudaMemcpyAsync(tabs, act_lut, 256, cudaMemcpyHostToDevice, p.d->stream),
                           "h2d"))
            return rc;
        if (int rc = check(cudaMemcpyAsync(tabs + 256, exp_lut, 256, cudaMemcpyHostToDevice,
                                           p.d->stream),
                           "h2d"))
            return rc;
        p.dout = dout;
        return hexcuda_decoder_block_i8(p.slot, dX, dW1, db1, reinterpret_cast<const int8_t *>(tabs),
                                        dW2, db2, tabs + 256, dout, S, D, Dff);
    });
}

HX_EXPORT int hexcuda_host_gemm_f16_ex(const uint16_t *A, const uint16_t *B, int b_transposed,
                                       const uint16_t *bias, const uint16_t *res, uint16_t *out,
                                       int act, int preround, float scale, int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_f16_ex: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_f16_ex", {A, B, out})) return rc;
    std::vector<const uint16_t *> dB(dev_count()), dbias(dev_count());
    // without a residual the second row input has no bytes and is not read
    return run_pipelined(
        M, {RowIn{A, 2 * (size_t)K, kSlotIn0}, RowIn{res, res ? 2 * (size_t)N : 0, kSlotIn3}},
        out, 2 * (size_t)N, pipe_chunk_bytes(kGemmChunkBytes),
        [&](Part &p) {
            const size_t s = (size_t)p.slot;
            dB[s] = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
            dbias[s] = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
            return (dB[s] && (!bias || dbias[s])) ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            const size_t s = (size_t)p.slot;
            return hexcuda_gemm_f16_ex(p.slot, (const uint16_t *)din[0], dB[s], b_transposed,
                                       dbias[s], res ? (const uint16_t *)din[1] : nullptr,
                                       (uint16_t *)dout, act, preround, scale, (int)nr, N, K);
        });
}

HX_EXPORT int hexcuda_host_gemm_i8_rq_ex(const int8_t *A, const int8_t *B, int b_transposed,
                                         const int32_t *bias, const int8_t *res, int8_t *out,
                                         int M, int N, int K, int32_t mult, int shift, int8_t zp,
                                         int relu) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_rq_ex: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i8_rq_ex", {A, B, out})) return rc;
    return run_sharded(M, out, (size_t)N, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        const int32_t *db = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
        const int8_t *dr = res ? stage_in(p.d, kSlotIn3, res + p.r0 * N, (size_t)(nr * N)) : nullptr;
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * N)));
        if (!dA || !dB || (bias && !db) || (res && !dr) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_i8_rq_ex(p.slot, dA, dB, b_transposed, db, dr, dout, (int)nr, N, K,
                                     mult, shift, zp, relu);
    });
}

HX_EXPORT int hexcuda_host_gemm_i8_acc(const void *A, int a_signed, const int8_t *B,
                                      int b_transposed, const int32_t *bias, const void *res,
                                      int res_kind, const void *lut, void *out, int store, int act,
                                      int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_acc: bad shape");
    if (store < HEXCUDA_HMX_STORE_I32 || store > HEXCUDA_HMX_STORE_ACC_I32 ||
        res_kind < HEXCUDA_HMX_RES_NONE || res_kind > HEXCUDA_HMX_RES_I8)
        return fail(HEXCUDA_ERR_ARG, "host_gemm_i8_acc: store %d / residual %d", store, res_kind);
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i8_acc", {A, B, out})) return rc;
    const bool has_lut = store == HEXCUDA_HMX_STORE_LUT_I32 || store == HEXCUDA_HMX_STORE_LUT_I8;
    const size_t osize = (store == HEXCUDA_HMX_STORE_I32 || store == HEXCUDA_HMX_STORE_LUT_I32 ||
                          store == HEXCUDA_HMX_STORE_ACC_I32) ? 4
                         : store == HEXCUDA_HMX_STORE_U16_FIELD ? 2 : 1;
    const size_t rsize = res_kind == HEXCUDA_HMX_RES_I32 ? 4 : 1;
    return run_sharded(M, out, (size_t)N * osize, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *dA = stage_in(p.d, kSlotIn0, reinterpret_cast<const uint8_t *>(A) + p.r0 * K,
                                     (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        const int32_t *db = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)N) : nullptr;
        const uint8_t *dr = res_kind ? stage_in(p.d, kSlotIn3,
                                                reinterpret_cast<const uint8_t *>(res) +
                                                    (size_t)p.r0 * N * rsize,
                                                (size_t)(nr * N) * rsize)
                                     : nullptr;
        const uint8_t *dl = has_lut ? stage_in(p.d, kSlotIn4, reinterpret_cast<const uint8_t *>(lut),
                                               store == HEXCUDA_HMX_STORE_LUT_I32 ? 1024 : 256)
                                    : nullptr;
        void *dout = scratch(p.d, kSlotOut, (size_t)(nr * N) * osize);
        if (!dA || !dB || (bias && !db) || (res_kind && !dr) || (has_lut && !dl) || !dout)
            return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_i8_acc(p.slot, dA, a_signed, dB, b_transposed, db, dr, res_kind, dl,
                                   dout, store, act, (int)nr, N, K);
    });
}

HX_EXPORT int hexcuda_host_ffn_relu_i8(const int8_t *A, const int8_t *W1, const int32_t *b1,
                                      const int8_t *W2, const int32_t *b2, int8_t *out, int M,
                                      int K, int V, int D, int32_t mult, int shift, int8_t zp) {
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "host_ffn_relu_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_ffn_relu_i8", {A, W1, b1, W2, b2, out})) return rc;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)K * V);
        const int32_t *db1 = stage_in(p.d, kSlotIn2, b1, (size_t)V);
        const int8_t *dW2 = stage_in(p.d, kSlotIn3, W2, (size_t)V * D);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D)));
        if (!dA || !dW1 || !db1 || !dW2 || !db2 || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_ffn_relu_i8(p.slot, dA, dW1, db1, dW2, db2, dout, (int)nr, K, V, D, mult,
                                   shift, zp);
    });
}

HX_EXPORT int hexcuda_host_gemm_hmx_s8u8(const int8_t *A, const uint8_t *B, void *out, int store,
                                         int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_hmx_s8u8: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_hmx_s8u8", {A, B, out})) return rc;
    const size_t osize = store == HEXCUDA_HMX_STORE_U16_FIELD ? 2
                         : (store == HEXCUDA_HMX_STORE_I32 || store == HEXCUDA_HMX_STORE_ACC_I32) ? 4 : 1;
    return run_sharded(M, out, (size_t)N * osize, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const uint8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        void *dout = scratch(p.d, kSlotOut, (size_t)(nr * N) * osize);
        if (!dA || !dB || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_hmx_s8u8(p.slot, dA, dB, dout, store, (int)nr, N, K);
    });
}

HX_EXPORT int hexcuda_host_gemm_f16_nt(const uint16_t *A, const uint16_t *Bt, uint16_t *out,
                                       int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_f16_nt: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_f16_nt", {A, Bt, out})) return rc;
    std::vector<const uint16_t *> dB(dev_count());
    return run_pipelined(
        M, {RowIn{A, 2 * (size_t)K, kSlotIn0}}, out, 2 * (size_t)N,
        pipe_chunk_bytes(kGemmChunkBytes),
        [&](Part &p) {
            dB[(size_t)p.slot] = stage_in(p.d, kSlotIn1, Bt, (size_t)N * K);
            return dB[(size_t)p.slot] ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            return hexcuda_gemm_f16_nt(p.slot, (const uint16_t *)din[0], dB[(size_t)p.slot],
                                       (uint16_t *)dout, (int)nr, N, K);
        });
}

HX_EXPORT int hexcuda_host_gemm_f16_nn(const uint16_t *A, const uint16_t *B, uint16_t *out, int M,
                                       int N, int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_f16_nn: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_f16_nn", {A, B, out})) return rc;
    std::vector<const uint16_t *> dB(dev_count());
    return run_pipelined(
        M, {RowIn{A, 2 * (size_t)K, kSlotIn0}}, out, 2 * (size_t)N,
        pipe_chunk_bytes(kGemmChunkBytes),
        [&](Part &p) {
            dB[(size_t)p.slot] = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
            return dB[(size_t)p.slot] ? HEXCUDA_OK : hexcuda_last_error();
        },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nr) {
            return hexcuda_gemm_f16_nn(p.slot, (const uint16_t *)din[0], dB[(size_t)p.slot],
                                       (uint16_t *)dout, (int)nr, N, K);
        });
}

HX_EXPORT int hexcuda_host_attn_f16(const uint16_t *Q, const uint16_t *K, const uint16_t *V,
                                    uint16_t *O, int BH, int SQ, int SK, int D, float scale,
                                    int causal) {
    if (BH < 0 || SQ < 0 || SK <= 0 || D <= 0)
        return fail(HEXCUDA_ERR_ARG, "host_attn_f16: BH=%d SQ=%d SK=%d D=%d", BH, SQ, SK, D);
    if (BH == 0 || SQ == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_attn_f16", {Q, K, V, O})) return rc;
    const size_t qh = (size_t)SQ * D, kh = (size_t)SK * D;
    return run_pipelined(
        BH, {RowIn{Q, 2 * qh, kSlotIn0}, RowIn{K, 2 * kh, kSlotIn1}, RowIn{V, 2 * kh, kSlotIn2}},
        O, 2 * qh, pipe_chunk_bytes(kGemmChunkBytes), [](Part &) { return HEXCUDA_OK; },
        [&](Part &p, const uint8_t *const *din, void *dout, int64_t nh) {
            return hexcuda_attn_f16(p.slot, (const uint16_t *)din[0], (const uint16_t *)din[1],
                                    (const uint16_t *)din[2], (uint16_t *)dout, (int)nh, SQ, SK,
                                    D, scale, causal);
        });
}

HX_EXPORT int hexcuda_host_online_softmax_step_f16(const uint16_t *scores, const uint16_t *V,
                                                   uint16_t *running_max, uint16_t *running_sum,
                                                   uint16_t *acc, int BLK, int D) {
    if (BLK <= 0 || D < 0)
        return fail(HEXCUDA_ERR_ARG, "host_online_softmax_step_f16: BLK=%d D=%d", BLK, D);
    if (int rc = null_check("host_online_softmax_step_f16", {scores, V, running_max, running_sum}))
        return rc;
    if (D > 0 && !acc) return fail(HEXCUDA_ERR_ARG, "host_online_softmax_step_f16: null acc");
    // state layout on the device: [max, sum, acc[0..D)]
    std::vector<uint16_t> state((size_t)D + 2);
    state[0] = *running_max;
    state[1] = *running_sum;
    std::copy(acc, acc + D, state.begin() + 2);
    std::vector<uint16_t> result(state.size());
    int rc = run_sharded(1, result.data(), 2 * state.size(), [&](Part &p) {
        const uint16_t *ds = stage_in(p.d, kSlotIn0, scores, (size_t)BLK);
        const uint16_t *dv = stage_in(p.d, kSlotIn1, V, (size_t)BLK * D);
        uint16_t *dst = stage_in(p.d, kSlotOut, state.data(), state.size());
        if (!ds || !dv || !dst) return hexcuda_last_error();
        p.dout = dst;
        return hexcuda_online_softmax_step_f16(p.slot, ds, dv, dst, dst + 1, dst + 2, BLK, D);
    });
    if (rc) return rc;
    *running_max = result[0];
    *running_sum = result[1];
    std::copy(result.begin() + 2, result.end(), acc);
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_host_minmax_ew(const void *a, const void *b, int32_t c, int elem, int op,
                                     void *out, int64_t n) {
    if (n < 0 || (elem != HEXCUDA_ELEM_I8 && elem != HEXCUDA_ELEM_U8 && elem != HEXCUDA_ELEM_I16))
        return fail(HEXCUDA_ERR_ARG, "host_minmax_ew: elem %d n %lld", elem, (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_minmax_ew", {a, out})) return rc;
    const size_t es = elem == HEXCUDA_ELEM_I16 ? 2 : 1;
    return run_sharded(n, out, es, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *da = stage_in(p.d, kSlotIn0, reinterpret_cast<const uint8_t *>(a) + p.r0 * es,
                                     (size_t)nr * es);
        const uint8_t *db = b ? stage_in(p.d, kSlotIn1, reinterpret_cast<const uint8_t *>(b) + p.r0 * es,
                                         (size_t)nr * es)
                              : nullptr;
        void *dout = scratch(p.d, kSlotOut, (size_t)nr * es);
        if (!da || (b && !db) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_minmax_ew(p.slot, da, db, c, elem, op, dout, nr);
    });
}

HX_EXPORT int hexcuda_host_group_sum_i8(const int8_t *a, int32_t *out, int64_t g, int w) {
    if (g < 0 || w < 1) return fail(HEXCUDA_ERR_ARG, "host_group_sum_i8: g %lld w %d", (long long)g, w);
    if (g == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_group_sum_i8", {a, out})) return rc;
    return run_sharded(g, out, 4, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *da = stage_in(p.d, kSlotIn0, a + p.r0 * w, (size_t)(nr * w));
        int32_t *dout = reinterpret_cast<int32_t *>(scratch(p.d, kSlotOut, (size_t)nr * 4));
        if (!da || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_group_sum_i8(p.slot, da, dout, nr, w);
    });
}

// a prefix scan: one device (the array as a single row)
HX_EXPORT int hexcuda_host_scan_max_i8(const int8_t *in, int8_t *out, int64_t n) {
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "host_scan_max_i8: n %lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_scan_max_i8", {in, out})) return rc;
    return run_sharded(1, out, (size_t)n, [&](Part &p) {
        const int8_t *din = stage_in(p.d, kSlotIn0, in, (size_t)n);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)n));
        if (!din || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_scan_max_i8(p.slot, din, dout, n);
    });
}

// groups (each with its H/G head planes) sharded over the devices
HX_EXPORT int hexcuda_host_head_group_reduce_i8(const int8_t *X, int8_t *Y, int H, int G,
                                                int64_t MN, int32_t mult, int shift) {
    if (H < 0 || G < 1 || MN < 0)
        return fail(HEXCUDA_ERR_ARG, "host_head_group_reduce_i8: H %d G %d MN %lld", H, G,
                    (long long)MN);
    if (MN == 0) return HEXCUDA_OK;
    const int HPG = H / G;
    if (int rc = null_check("host_head_group_reduce_i8", {HPG ? (const void *)X : Y, Y})) return rc;
    return run_sharded(G, Y, (size_t)MN, [&](Part &p) {
        const int64_t ng = p.r1 - p.r0;
        const int8_t *dx = HPG ? stage_in(p.d, kSlotIn0, X + p.r0 * HPG * MN, (size_t)(ng * HPG * MN))
                               : nullptr;
        int8_t *dy = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(ng * MN)));
        if ((HPG && !dx) || !dy) return hexcuda_last_error();
        p.dout = dy;
        // the shard's groups: H' = ng * HPG heads in ng groups
        return hexcuda_head_group_reduce_i8(p.slot, dx, dy, (int)(ng * HPG), (int)ng, MN, mult,
                                            shift);
    });
}

// Rows sharded over the devices; a gathered layernorm (idx) replicates the
// table x (xrows rows) and shards idx; per-row affine operands are sharded
// with their rows, shared ones replicated.
HX_EXPORT int hexcuda_host_layernorm_lut_i8(const int8_t *x, int xrows, const int32_t *idx,
                                            const int8_t *res, int8_t *out, int R, int W,
                                            const int8_t *gamma, const int8_t *beta,
                                            const uint8_t *inv_lut, int affine) {
    if (R < 0 || W < 1 || (idx && xrows < 1) || affine < HEXCUDA_LN_AFFINE_SHARED ||
        affine > HEXCUDA_LN_RMS_SHARED)
        return fail(HEXCUDA_ERR_ARG, "host_layernorm_lut_i8: R %d W %d affine %d", R, W, affine);
    if (R == 0) return HEXCUDA_OK;
    const bool rms = affine == HEXCUDA_LN_RMS_SHARED;
    if (int rc = null_check("host_layernorm_lut_i8", {x, out, gamma, rms ? gamma : beta, inv_lut}))
        return rc;
    return run_sharded(R, out, (size_t)W, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dx = idx ? stage_in(p.d, kSlotIn0, x, (size_t)xrows * W)
                               : stage_in(p.d, kSlotIn0, x + p.r0 * W, (size_t)(nr * W));
        const int32_t *di = idx ? stage_in(p.d, kSlotIn1, idx + p.r0, (size_t)nr) : nullptr;
        const int8_t *dr = res ? stage_in(p.d, kSlotIn2, res + p.r0 * W, (size_t)(nr * W)) : nullptr;
        int64_t g0 = 0, gn = W, l0 = 0, ln = 256;
        if (affine == HEXCUDA_LN_AFFINE_ROWWISE) g0 = p.r0 * W, gn = nr * W;
        if (affine == HEXCUDA_LN_AFFINE_PER_ROW) g0 = p.r0, gn = nr, l0 = p.r0 * 256, ln = nr * 256;
        const int8_t *dg = stage_in(p.d, kSlotIn3, gamma + g0, (size_t)gn);
        const int8_t *db = rms ? nullptr : stage_in(p.d, kSlotIn4, beta + g0, (size_t)gn);
        const uint8_t *dl = stage_in(p.d, kSlotIn5, inv_lut + l0, (size_t)ln);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * W)));
        if (!dx || (idx && !di) || (res && !dr) || !dg || (!rms && !db) || !dl || !dout)
            return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_layernorm_lut_i8(p.slot, dx, di, dr, dout, (int)nr, W, dg, db, dl, affine);
    });
}

HX_EXPORT int hexcuda_host_layernorm_lut_i16(const int16_t *x, int16_t *out, int R, int C,
                                             const int16_t *gamma, const int16_t *beta,
                                             const uint16_t *inv_lut, int order) {
    if (R < 0 || C < 1 || (order != 0 && order != 1))
        return fail(HEXCUDA_ERR_ARG, "host_layernorm_lut_i16: R %d C %d order %d", R, C, order);
    if (R == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_layernorm_lut_i16", {x, out, gamma, beta, inv_lut})) return rc;
    return run_sharded(R, out, (size_t)C * 2, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int16_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const int64_t g0 = order ? p.r0 : 0, gn = order ? nr : C;
        const int16_t *dg = stage_in(p.d, kSlotIn1, gamma + g0, (size_t)gn);
        const int16_t *db = stage_in(p.d, kSlotIn2, beta + g0, (size_t)gn);
        const uint16_t *dl = stage_in(p.d, kSlotIn3, inv_lut, 256);
        int16_t *dout = reinterpret_cast<int16_t *>(scratch(p.d, kSlotOut, (size_t)(nr * C) * 2));
        if (!dx || !dg || !db || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_layernorm_lut_i16(p.slot, dx, dout, (int)nr, C, dg, db, dl, order);
    });
}

HX_EXPORT int hexcuda_host_lut_softmax_u8(const int8_t *x, uint8_t *out, int R, int C,
                                          const uint8_t *exp_lut, const uint16_t *recip_lut) {
    if (R < 0 || C < 1) return fail(HEXCUDA_ERR_ARG, "host_lut_softmax_u8: R %d C %d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_lut_softmax_u8", {x, out, exp_lut})) return rc;
    return run_sharded(R, out, (size_t)C, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const uint8_t *dl = stage_in(p.d, kSlotIn1, exp_lut, 256);
        const uint16_t *dr = recip_lut ? stage_in(p.d, kSlotIn2, recip_lut, 256) : nullptr;
        uint8_t *dout = reinterpret_cast<uint8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * C)));
        if (!dx || !dl || (recip_lut && !dr) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_lut_softmax_u8(p.slot, dx, dout, (int)nr, C, dl, dr);
    });
}

HX_EXPORT int hexcuda_host_lut_softmax_i16(const int16_t *x, int16_t *out, int R, int C,
                                           const uint16_t *exp_lut) {
    if (R < 0 || C < 1) return fail(HEXCUDA_ERR_ARG, "host_lut_softmax_i16: R %d C %d", R, C);
    if (R == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_lut_softmax_i16", {x, out, exp_lut})) return rc;
    return run_sharded(R, out, (size_t)C * 2, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int16_t *dx = stage_in(p.d, kSlotIn0, x + p.r0 * C, (size_t)(nr * C));
        const uint16_t *dl = stage_in(p.d, kSlotIn1, exp_lut, 256);
        int16_t *dout = reinterpret_cast<int16_t *>(scratch(p.d, kSlotOut, (size_t)(nr * C) * 2));
        if (!dx || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_lut_softmax_i16(p.slot, dx, dout, (int)nr, C, dl);
    });
}

HX_EXPORT int hexcuda_host_requant_i16(const int32_t *a, int16_t *out, int64_t n, int32_t mult,
                                       int shift) {
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "host_requant_i16: n %lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_requant_i16", {a, out})) return rc;
    return run_sharded(n, out, 2, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int32_t *da = stage_in(p.d, kSlotIn0, a + p.r0, (size_t)nr);
        int16_t *dout = reinterpret_cast<int16_t *>(scratch(p.d, kSlotOut, (size_t)nr * 2));
        if (!da || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_requant_i16(p.slot, da, dout, nr, mult, shift);
    });
}

// channels are fixed fractions of n: one device
HX_EXPORT int hexcuda_host_norm_requant_i8(const int8_t *a, int8_t *out, int64_t n, int nch,
                                           const int32_t *nmult, const int *nshift, int32_t mult,
                                           int shift, int zp) {
    if (n < 0 || nch < 1) return fail(HEXCUDA_ERR_ARG, "host_norm_requant_i8: n %lld", (long long)n);
    const int64_t used = n / nch * nch;
    if (used == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_norm_requant_i8", {a, out, nmult, nshift})) return rc;
    return run_sharded(1, out, (size_t)used, [&](Part &p) {
        const int8_t *da = stage_in(p.d, kSlotIn0, a, (size_t)used);
        const int32_t *dm = stage_in(p.d, kSlotIn1, nmult, (size_t)nch);
        const int *ds = stage_in(p.d, kSlotIn2, nshift, (size_t)nch);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)used));
        if (!da || !dm || !ds || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_norm_requant_i8(p.slot, da, dout, used, nch, dm, ds, mult, shift, zp);
    });
}

HX_EXPORT int hexcuda_host_gemm_softmax_u8(const int8_t *A, const int8_t *B, int b_transposed,
                                           const uint8_t *exp_lut, uint8_t *out, int M, int N,
                                           int K, int requant, int32_t mult, int shift) {
    if (M < 0 || N < 1 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_softmax_u8: bad shape");
    if (M == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_softmax_u8", {A, B, exp_lut, out})) return rc;
    return run_sharded(M, out, (size_t)N, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        const uint8_t *dl = stage_in(p.d, kSlotIn2, exp_lut, 256);
        uint8_t *dout = reinterpret_cast<uint8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * N)));
        if (!dA || !dB || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gemm_softmax_u8(p.slot, dA, dB, b_transposed, dl, dout, (int)nr, N, K,
                                       requant, mult, shift);
    });
}

HX_EXPORT int hexcuda_host_gelu_ffn_residual_i8(const int8_t *x, const int8_t *W1, const int32_t *b1,
                                                const int8_t *gelu_lut, const int8_t *W2,
                                                const int32_t *b2, const int8_t *x_res,
                                                const int8_t *gamma, const int8_t *beta,
                                                const uint8_t *inv_lut, int8_t *out, int M, int K,
                                                int V, int D) {
    if (M < 0 || K < 0 || V < 0 || D < 1) return fail(HEXCUDA_ERR_ARG, "host_gelu_ffn_residual_i8: bad shape");
    if (M == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gelu_ffn_residual_i8",
                            {x, W1, b1, gelu_lut, W2, b2, x_res, gamma, beta, inv_lut, out}))
        return rc;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        // 8 staged operands: the weights and tables share the input slots
        // with the row-sharded activations through one packed buffer
        const size_t nx = (size_t)(nr * K), nw1 = (size_t)K * V, nw2 = (size_t)V * D,
                     nres = (size_t)(nr * D);
        auto r16 = [](size_t b) { return (b + 15) / 16 * 16; };
        uint8_t *pk = reinterpret_cast<uint8_t *>(
            scratch(p.d, kSlotIn0, r16(nx) + r16(nw1) + r16(nw2) + r16(nres) + 2 * r16((size_t)D) + 512));
        int32_t *dbias = reinterpret_cast<int32_t *>(scratch(p.d, kSlotIn1, 4 * ((size_t)V + D)));
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, nres));
        if (!pk || !dbias || !dout) return hexcuda_last_error();
        size_t off = 0;
        auto put = [&](const void *src, size_t bytes) -> uint8_t * {
            uint8_t *dst = pk + off;
            off += (bytes + 15) / 16 * 16;
            if (bytes && check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, p.d->stream), "h2d"))
                return nullptr;
            return dst;
        };
        const int8_t *dx = reinterpret_cast<const int8_t *>(put(x + p.r0 * K, nx));
        const int8_t *dw1 = reinterpret_cast<const int8_t *>(put(W1, nw1));
        const int8_t *dw2 = reinterpret_cast<const int8_t *>(put(W2, nw2));
        const int8_t *dres = reinterpret_cast<const int8_t *>(put(x_res + p.r0 * D, nres));
        const int8_t *dg = reinterpret_cast<const int8_t *>(put(gamma, (size_t)D));
        const int8_t *dbt = reinterpret_cast<const int8_t *>(put(beta, (size_t)D));
        const int8_t *dgl = reinterpret_cast<const int8_t *>(put(gelu_lut, 256));
        const uint8_t *dil = put(inv_lut, 256);
        if (check(cudaMemcpyAsync(dbias, b1, 4 * (size_t)V, cudaMemcpyHostToDevice, p.d->stream), "h2d") ||
            check(cudaMemcpyAsync(dbias + V, b2, 4 * (size_t)D, cudaMemcpyHostToDevice, p.d->stream), "h2d"))
            return hexcuda_last_error();
        if (!dx || !dw1 || !dw2 || !dres || !dg || !dbt || !dgl || !dil) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gelu_ffn_residual_i8(p.slot, dx, dw1, dbias, dgl, dw2, dbias + V, dres, dg, dbt,
                                            dil, dout, (int)nr, K, V, D);
    });
}

HX_EXPORT int hexcuda_host_group_dot_i8(const int8_t *a, const int8_t *b, int32_t *out, int64_t g,
                                        int w) {
    if (g < 0 || w < 1) return fail(HEXCUDA_ERR_ARG, "host_group_dot_i8: g %lld w %d", (long long)g, w);
    if (g == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_group_dot_i8", {a, b, out})) return rc;
    return run_sharded(g, out, 4, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *da = stage_in(p.d, kSlotIn0, a + p.r0 * w, (size_t)(nr * w));
        const int8_t *db = stage_in(p.d, kSlotIn1, b + p.r0 * w, (size_t)(nr * w));
        int32_t *dout = reinterpret_cast<int32_t *>(scratch(p.d, kSlotOut, (size_t)nr * 4));
        if (!da || !db || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_group_dot_i8(p.slot, da, db, dout, nr, w);
    });
}

HX_EXPORT int hexcuda_host_gate_mul_requant_i8(const int8_t *gate, const int8_t *up,
                                               const int8_t *lut, int8_t *out, int64_t n,
                                               int32_t mult, int shift) {
    if (n < 0) return fail(HEXCUDA_ERR_ARG, "host_gate_mul_requant_i8: n %lld", (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gate_mul_requant_i8", {gate, up, lut, out})) return rc;
    return run_sharded(n, out, 1, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dg = stage_in(p.d, kSlotIn0, gate + p.r0, (size_t)nr);
        const int8_t *du = stage_in(p.d, kSlotIn1, up + p.r0, (size_t)nr);
        const int8_t *dl = stage_in(p.d, kSlotIn2, lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)nr));
        if (!dg || !du || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_gate_mul_requant_i8(p.slot, dg, du, dl, dout, nr, mult, shift);
    });
}

HX_EXPORT int hexcuda_host_ffn_lut_i8(const int8_t *A, const int8_t *W1, const int32_t *b1,
                                      const int8_t *act_lut, const int8_t *W2, const int32_t *b2,
                                      int8_t *out, int M, int K, int V, int D, int32_t mult,
                                      int shift, int8_t zp) {
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "host_ffn_lut_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_ffn_lut_i8", {A, W1, b1, act_lut, W2, b2, out})) return rc;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)K * V);
        const int32_t *db1 = stage_in(p.d, kSlotIn2, b1, (size_t)V);
        const int8_t *dW2 = stage_in(p.d, kSlotIn3, W2, (size_t)V * D);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        const int8_t *dl = stage_in(p.d, kSlotIn5, act_lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D)));
        if (!dA || !dW1 || !db1 || !dW2 || !db2 || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_ffn_lut_i8(p.slot, dA, dW1, db1, dl, dW2, db2, dout, (int)nr, K, V, D, mult,
                                  shift, zp);
    });
}

// Heads are split over the devices; each shard's K cache rows come back
// through run_sharded, its V cache rows by a copy queued after the kernel.
HX_EXPORT int hexcuda_host_kv_cache_update_i8(int8_t *k_cache, int8_t *v_cache,
                                              const int8_t *k_new, const int8_t *v_new, int pos,
                                              int heads, int cache_len, int head_dim) {
    if (heads < 0 || cache_len < 1 || head_dim < 0 || pos < 0 || pos >= cache_len)
        return fail(HEXCUDA_ERR_ARG, "host_kv_cache_update_i8: pos %d heads %d cache_len %d head_dim %d",
                    pos, heads, cache_len, head_dim);
    if (heads == 0 || head_dim == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_kv_cache_update_i8", {k_cache, v_cache, k_new, v_new})) return rc;
    const size_t plane = (size_t)cache_len * head_dim;
    return run_sharded(heads, k_cache, plane, [&](Part &p) {
        const int64_t nh = p.r1 - p.r0;
        int8_t *dk = stage_in(p.d, kSlotIn0, k_cache + p.r0 * plane, (size_t)nh * plane);
        int8_t *dv = stage_in(p.d, kSlotIn1, v_cache + p.r0 * plane, (size_t)nh * plane);
        const int8_t *dkn = stage_in(p.d, kSlotIn2, k_new + p.r0 * head_dim, (size_t)(nh * head_dim));
        const int8_t *dvn = stage_in(p.d, kSlotIn3, v_new + p.r0 * head_dim, (size_t)(nh * head_dim));
        if (!dk || !dv || !dkn || !dvn) return hexcuda_last_error();
        if (int rc = hexcuda_kv_cache_update_i8(p.slot, dk, dv, dkn, dvn, pos, (int)nh, cache_len,
                                                head_dim))
            return rc;
        p.dout = dk;
        return check(cudaMemcpyAsync(v_cache + p.r0 * plane, dv, (size_t)nh * plane,
                                     cudaMemcpyDeviceToHost, p.d->stream),
                     "d2h (V cache)");
    });
}

HX_EXPORT int hexcuda_host_rope_pair_f16(const uint16_t *x, const uint16_t *cos_t,
                                         const uint16_t *sin_t, uint16_t *out, int64_t n_pairs) {
    if (n_pairs < 0)
        return fail(HEXCUDA_ERR_ARG, "host_rope_pair_f16: n_pairs %lld", (long long)n_pairs);
    if (n_pairs == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_rope_pair_f16", {x, cos_t, sin_t, out})) return rc;
    return run_sharded(n_pairs, out, 4, [&](Part &p) {
        const int64_t np = p.r1 - p.r0;
        const uint16_t *dx = stage_in(p.d, kSlotIn0, x + 2 * p.r0, (size_t)(2 * np));
        const uint16_t *dc = stage_in(p.d, kSlotIn1, cos_t + p.r0, (size_t)np);
        const uint16_t *ds = stage_in(p.d, kSlotIn2, sin_t + p.r0, (size_t)np);
        uint16_t *dout = reinterpret_cast<uint16_t *>(scratch(p.d, kSlotOut, (size_t)np * 4));
        if (!dx || !dc || !ds || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_rope_pair_f16(p.slot, dx, dc, ds, dout, np);
    });
}

HX_EXPORT int hexcuda_host_ffn_hmx_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                      const int8_t *W2, const int32_t *b2, int8_t *out, int M,
                                      int D, int Dff, int sh1, int sh2) {
    if (M < 0 || D < 0 || Dff < 0) return fail(HEXCUDA_ERR_ARG, "host_ffn_hmx_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_ffn_hmx_i8", {X, W1, b1, W2, b2, out})) return rc;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *dX = stage_in(p.d, kSlotIn0, X + p.r0 * D, (size_t)(nr * D));
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)D * Dff);
        const int32_t *db1 = stage_in(p.d, kSlotIn2, b1, (size_t)Dff);
        const int8_t *dW2 = stage_in(p.d, kSlotIn3, W2, (size_t)Dff * D);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D)));
        if (!dX || !dW1 || !db1 || !dW2 || !db2 || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_ffn_hmx_i8(p.slot, dX, dW1, db1, dW2, db2, dout, (int)nr, D, Dff, sh1, sh2);
    });
}

// The gate and up weights share one staging slot (two halves).
HX_EXPORT int hexcuda_host_ffn_swiglu_hmx_i8(const uint8_t *X, const int8_t *Wg, const int8_t *Wu,
                                             const int8_t *Wd, const int32_t *bd,
                                             const uint8_t *silu_lut, int8_t *out, int M, int D,
                                             int Dff, int sg, int su, int sh, int zp, int so) {
    if (M < 0 || D < 0 || Dff < 0) return fail(HEXCUDA_ERR_ARG, "host_ffn_swiglu_hmx_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_ffn_swiglu_hmx_i8", {X, Wg, Wu, Wd, bd, silu_lut, out})) return rc;
    const size_t wsz = (size_t)D * Dff, wpad = (wsz + 15) & ~(size_t)15;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *dX = stage_in(p.d, kSlotIn0, X + p.r0 * D, (size_t)(nr * D));
        int8_t *dW = reinterpret_cast<int8_t *>(scratch(p.d, kSlotIn1, 2 * wpad + 16));
        const int8_t *dWd = stage_in(p.d, kSlotIn2, Wd, wsz);
        const int32_t *dbd = stage_in(p.d, kSlotIn3, bd, (size_t)D);
        const uint8_t *dl = stage_in(p.d, kSlotIn4, silu_lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D)));
        if (!dX || !dW || !dWd || !dbd || !dl || !dout) return hexcuda_last_error();
        if (wsz) {
            if (int rc = check(cudaMemcpyAsync(dW, Wg, wsz, cudaMemcpyHostToDevice, p.d->stream), "h2d"))
                return rc;
            if (int rc = check(cudaMemcpyAsync(dW + wpad, Wu, wsz, cudaMemcpyHostToDevice, p.d->stream),
                               "h2d"))
                return rc;
        }
        p.dout = dout;
        return hexcuda_ffn_swiglu_hmx_i8(p.slot, dX, dW, dW + wpad, dWd, dbd, dl, dout, (int)nr, D, Dff,
                                         sg, su, sh, zp, so);
    });
}

HX_EXPORT int hexcuda_host_encoder_block_i8(const uint8_t *X, const int8_t *W1, const int32_t *b1,
                                            const int8_t *W2, const int32_t *b2,
                                            const uint8_t *exp_lut, int8_t *out, int S, int D,
                                            int Dff) {
    if (S < 0 || D < 0 || Dff < 0) return fail(HEXCUDA_ERR_ARG, "host_encoder_block_i8: bad shape");
    if (S == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_encoder_block_i8", {X, W1, b1, W2, b2, exp_lut, out})) return rc;
    return run_sharded(1, out, (size_t)S * D, [&](Part &p) {
        const uint8_t *dX = stage_in(p.d, kSlotIn0, X, (size_t)S * D);
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)D * Dff);
        const int8_t *dW2 = stage_in(p.d, kSlotIn2, W2, (size_t)Dff * D);
        const int32_t *db1 = stage_in(p.d, kSlotIn3, b1, (size_t)Dff);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        const uint8_t *dl = stage_in(p.d, kSlotIn5, exp_lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)S * D));
        if (!dX || !dW1 || !dW2 || !db1 || !db2 || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_encoder_block_i8(p.slot, dX, dW1, db1, dW2, db2, dl, dout, S, D, Dff);
    });
}

HX_EXPORT int hexcuda_host_affine_ew(const void *in, int elem_in, void *out, int elem_out, int64_t n,
                                     int32_t zp_in, int32_t mult, int64_t add, int shift, int round,
                                     int wrap32, int zp_out, int32_t lo, int32_t hi) {
    if (elem_in < HEXCUDA_ELEM_I8 || elem_in > HEXCUDA_ELEM_I32 || elem_out < HEXCUDA_ELEM_I8 ||
        elem_out > HEXCUDA_ELEM_I32 || n < 0)
        return fail(HEXCUDA_ERR_ARG, "host_affine_ew: elem %d -> %d n %lld", elem_in, elem_out,
                    (long long)n);
    if (n == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_affine_ew", {in, out})) return rc;
    auto esz = [](int e) { return e == HEXCUDA_ELEM_I32 ? (size_t)4 : (e == HEXCUDA_ELEM_I16 ? (size_t)2 : (size_t)1); };
    const size_t ei = esz(elem_in), eo = esz(elem_out);
    return run_sharded(n, out, eo, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const uint8_t *din = stage_in(p.d, kSlotIn0, reinterpret_cast<const uint8_t *>(in) + p.r0 * ei,
                                      (size_t)nr * ei);
        void *dout = scratch(p.d, kSlotOut, (size_t)nr * eo);
        if (!din || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_affine_ew(p.slot, din, elem_in, dout, elem_out, nr, zp_in, mult, add, shift,
                                 round, wrap32, zp_out, lo, hi);
    });
}

HX_EXPORT int hexcuda_host_gemm_i16(const int16_t *A, const int16_t *B, int32_t *C, int M, int N,
                                    int K) {
    if (M < 0 || N < 0 || K < 0) return fail(HEXCUDA_ERR_ARG, "host_gemm_i16: bad shape");
    if (M == 0 || N == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_gemm_i16", {A, B, C})) return rc;
    return run_sharded(M, C, (size_t)N * 4, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int16_t *dA = stage_in(p.d, kSlotIn0, A + p.r0 * K, (size_t)(nr * K));
        const int16_t *dB = stage_in(p.d, kSlotIn1, B, (size_t)K * N);
        int32_t *dC = reinterpret_cast<int32_t *>(scratch(p.d, kSlotOut, (size_t)nr * N * 4));
        if ((K && (!dA || !dB)) || !dC) return hexcuda_last_error();
        p.dout = dC;
        return hexcuda_gemm_i16(p.slot, dA, dB, dC, (int)nr, N, K);
    });
}

HX_EXPORT int hexcuda_host_mix_mlp_i8(const int8_t *X, const int8_t *W1, const int32_t *b1,
                                      const int8_t *lut, const int8_t *W2, const int32_t *b2,
                                      int8_t *out, int M, int K, int V, int D, int32_t mult1,
                                      int shift1, int32_t mult2, int shift2) {
    if (M < 0 || K < 0 || V < 0 || D < 0) return fail(HEXCUDA_ERR_ARG, "host_mix_mlp_i8: bad shape");
    if (M == 0 || D == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_mix_mlp_i8", {X, W1, b1, W2, b2, out})) return rc;
    return run_sharded(M, out, (size_t)D, [&](Part &p) {
        const int64_t nr = p.r1 - p.r0;
        const int8_t *dX = stage_in(p.d, kSlotIn0, X + p.r0 * K, (size_t)(nr * K));
        const int8_t *dW1 = stage_in(p.d, kSlotIn1, W1, (size_t)V * K);
        const int32_t *db1 = stage_in(p.d, kSlotIn2, b1, (size_t)V);
        const int8_t *dW2 = stage_in(p.d, kSlotIn3, W2, (size_t)D * V);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)D);
        const int8_t *dl = lut ? stage_in(p.d, kSlotIn5, lut, 256) : nullptr;
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)(nr * D)));
        if (!dX || !dW1 || !db1 || !dW2 || !db2 || (lut && !dl) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_mix_mlp_i8(p.slot, dX, dW1, db1, dl, dW2, db2, dout, (int)nr, K, V, D, mult1,
                                  shift1, mult2, shift2);
    });
}

HX_EXPORT int hexcuda_host_token_mix_i8(const int8_t *X, const int8_t *W, const int32_t *b,
                                        const int8_t *W2, const int32_t *b2, int8_t *out, int T,
                                        int C, int DM, int32_t mult1, int shift1, int32_t mult2,
                                        int shift2) {
    if (T < 0 || C < 0 || DM < 0) return fail(HEXCUDA_ERR_ARG, "host_token_mix_i8: bad shape");
    if (T == 0 || C == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_token_mix_i8", {X, W, b, W2, b2, out})) return rc;
    return run_sharded(1, out, (size_t)T * C, [&](Part &p) {
        const int8_t *dX = stage_in(p.d, kSlotIn0, X, (size_t)T * C);
        const int8_t *dW = stage_in(p.d, kSlotIn1, W, (size_t)DM * T);
        const int32_t *db = stage_in(p.d, kSlotIn2, b, (size_t)DM);
        const int8_t *dW2 = stage_in(p.d, kSlotIn3, W2, (size_t)T * DM);
        const int32_t *db2 = stage_in(p.d, kSlotIn4, b2, (size_t)T);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)T * C));
        if (!dX || !dW || !db || !dW2 || !db2 || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_token_mix_i8(p.slot, dX, dW, db, dW2, db2, dout, T, C, DM, mult1, shift1, mult2,
                                    shift2);
    });
}

HX_EXPORT int hexcuda_host_rnn_cell_i8(const int8_t *Wx, const int8_t *Wh, const int32_t *b,
                                       const int8_t *x, const int8_t *h_prev, int8_t *h_t, int H,
                                       int I, int32_t mult, int shift, int8_t zp,
                                       const int8_t *tanh_lut) {
    if (H < 0 || I < 0) return fail(HEXCUDA_ERR_ARG, "host_rnn_cell_i8: H %d I %d", H, I);
    if (H == 0) return HEXCUDA_OK;
    if (int rc = null_check("host_rnn_cell_i8", {Wh, b, h_prev, h_t, tanh_lut})) return rc;
    if (I > 0 && (!Wx || !x)) return fail(HEXCUDA_ERR_ARG, "host_rnn_cell_i8: null pointer");
    return run_sharded(1, h_t, (size_t)H, [&](Part &p) {
        const int8_t *dWx = I ? stage_in(p.d, kSlotIn0, Wx, (size_t)H * I) : nullptr;
        const int8_t *dWh = stage_in(p.d, kSlotIn1, Wh, (size_t)H * H);
        const int32_t *db = stage_in(p.d, kSlotIn2, b, (size_t)H);
        const int8_t *dx = I ? stage_in(p.d, kSlotIn3, x, (size_t)I) : nullptr;
        const int8_t *dh = stage_in(p.d, kSlotIn4, h_prev, (size_t)H);
        const int8_t *dl = stage_in(p.d, kSlotIn5, tanh_lut, 256);
        int8_t *dout = reinterpret_cast<int8_t *>(scratch(p.d, kSlotOut, (size_t)H));
        if ((I && (!dWx || !dx)) || !dWh || !db || !dh || !dl || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_rnn_cell_i8(p.slot, dWx, dWh, db, dx, dh, dout, H, I, mult, shift, zp, dl);
    });
}

HX_EXPORT int hexcuda_host_conv2d_hmx(const uint8_t *in, const int8_t *W, const int32_t *bias,
                                      void *out, int store, int act, int c_in, int ih, int iw,
                                      int c_out, int kh, int kw, int stride) {
    if (c_in < 1 || c_out < 1 || kh < 1 || kw < 1 || stride < 1 || ih < kh || iw < kw)
        return fail(HEXCUDA_ERR_ARG, "host_conv2d_hmx: bad shape");
    if (int rc = null_check("host_conv2d_hmx", {in, W, out})) return rc;
    const int oh = (ih - kh) / stride + 1, ow = (iw - kw) / stride + 1;
    const size_t es = store == HEXCUDA_HMX_STORE_I32 ? 4 : (store == HEXCUDA_HMX_STORE_U16_FIELD ? 2 : 1);
    const size_t obytes = (size_t)c_out * oh * ow * es;
    return run_sharded(1, out, obytes, [&](Part &p) {
        const uint8_t *din = stage_in(p.d, kSlotIn0, in, (size_t)c_in * ih * iw);
        const int8_t *dW = stage_in(p.d, kSlotIn1, W, (size_t)c_out * c_in * kh * kw);
        const int32_t *db = bias ? stage_in(p.d, kSlotIn2, bias, (size_t)c_out) : nullptr;
        void *dout = scratch(p.d, kSlotOut, obytes);
        if (!din || !dW || (bias && !db) || !dout) return hexcuda_last_error();
        p.dout = dout;
        return hexcuda_conv2d_hmx(p.slot, din, dW, db, dout, store, act, c_in, ih, iw, c_out, kh, kw,
                                  stride);
    });
}
