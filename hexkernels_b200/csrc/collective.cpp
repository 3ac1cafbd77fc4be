// collective.cpp -- replicated outputs: an NCCL all-gather of row shards over
// NVLink, either in one process over every initialised device or across
// processes (one GPU per process).
//
// Every operator shards its rows (M rows, B*H heads, elements) into contiguous
// parts, part i owning [rows*i/n, rows*(i+1)/n).  When a caller asks for the
// output on every GPU, the parts are gathered in place of a host round trip:
//   * equal parts (rows divisible by n): one ncclAllGather per device;
//   * ragged parts: one ncclBroadcast per owning part, all inside one NCCL
//     group, each landing at that part's row offset of every replica.
// Both move exactly the bytes of the other parts into each device's replica;
// nothing else crosses NVLink and no kernel reads a peer's memory.
//
// NCCL is opened with dlopen on first use, so programs that never ask for a
// replicated output (the corpus harnesses) do not depend on it; in a process
// that already loaded NCCL (torch.distributed) the same library is reused.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <vector>

#include "hx_internal.h"

namespace hx {
namespace {

struct NcclApi {
    bool tried = false, ok = false;
    int version = 0;
    ncclResult_t (*GetVersion)(int *);
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommInitAll)(ncclComm_t *, int, const int *);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t);
    ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t,
                              cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
};

NcclApi g_nccl;

template <typename F>
bool sym(void *h, const char *name, F &fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

bool nccl_load() {
    if (g_nccl.tried) return g_nccl.ok;
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        fail(HEXCUDA_ERR_CUDA, "replicated output needs NCCL: dlopen(libnccl.so.2): %s", dlerror());
        return false;
    }
    NcclApi &a = g_nccl;
    bool ok = sym(h, "ncclGetVersion", a.GetVersion) && sym(h, "ncclGetUniqueId", a.GetUniqueId) &&
              sym(h, "ncclCommInitRank", a.CommInitRank) &&
              sym(h, "ncclCommInitAll", a.CommInitAll) &&
              sym(h, "ncclCommDestroy", a.CommDestroy) && sym(h, "ncclAllGather", a.AllGather) &&
              sym(h, "ncclBroadcast", a.Broadcast) && sym(h, "ncclGroupStart", a.GroupStart) &&
              sym(h, "ncclGroupEnd", a.GroupEnd) &&
              sym(h, "ncclGetErrorString", a.GetErrorString);
    if (!ok) {
        fail(HEXCUDA_ERR_CUDA, "libnccl.so.2 lacks a required symbol");
        return false;
    }
    a.GetVersion(&a.version);
    a.ok = true;
    return true;
}

int ncheck(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return HEXCUDA_OK;
    return fail(HEXCUDA_ERR_CUDA, "%s: %s (nccl %d)", what, g_nccl.GetErrorString(r), (int)r);
}

// Communicator modes: none, one process over all its initialised devices
// (ncclCommInitAll), or one rank of a multi-process group (device slot 0).
enum CommMode { kCommNone = 0, kCommLocal = 1, kCommRank = 2 };
int g_mode = kCommNone;
int g_nranks = 0, g_rank = -1;
bool g_replicate = false;
float g_coll_ms = -1.0f;

// Per initialised device: its communicator and the collective's events.
struct CollDev {
    int ordinal = -1;
    ncclComm_t comm = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    void *replica = nullptr;
    size_t replica_bytes = 0;
};
std::vector<CollDev> g_cd;

void destroy_comms() {
    for (auto &c : g_cd) {
        if (c.ordinal >= 0) cudaSetDevice(c.ordinal);
        if (c.comm && g_nccl.ok) g_nccl.CommDestroy(c.comm);
        if (c.e0) cudaEventDestroy(c.e0);
        if (c.e1) cudaEventDestroy(c.e1);
    }
    g_cd.clear();
    g_mode = kCommNone;
    g_nranks = 0;
    g_rank = -1;
}

int make_events(CollDev &c) {
    if (int rc = check(cudaEventCreate(&c.e0), "cudaEventCreate(collective)")) return rc;
    return check(cudaEventCreate(&c.e1), "cudaEventCreate(collective)");
}

// The in-process communicator over every initialised device (rebuilt when
// the device set changed).
int ensure_local_comms() {
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const int n = ndev();
    if (g_mode == kCommLocal && (int)g_cd.size() == n) {
        bool same = true;
        for (int i = 0; i < n; i++) same = same && g_cd[(size_t)i].ordinal == hexcuda_device_ordinal(i);
        if (same) return HEXCUDA_OK;
    }
    if (g_mode == kCommRank)
        return fail(HEXCUDA_ERR_ARG,
                    "this process joined a multi-process group (hexcuda_comm_init_rank); "
                    "in-process gathers are not available");
    destroy_comms();
    if (!nccl_load()) return hexcuda_last_error();
    std::vector<int> ords((size_t)n);
    for (int i = 0; i < n; i++) ords[(size_t)i] = hexcuda_device_ordinal(i);
    std::vector<ncclComm_t> comms((size_t)n, nullptr);
    if (int rc = ncheck(g_nccl.CommInitAll(comms.data(), n, ords.data()), "ncclCommInitAll"))
        return rc;
    g_cd.assign((size_t)n, CollDev());
    for (int i = 0; i < n; i++) {
        CollDev &c = g_cd[(size_t)i];
        c.ordinal = ords[(size_t)i];
        c.comm = comms[(size_t)i];
        if (int rc = check(cudaSetDevice(c.ordinal), "cudaSetDevice")) return rc;
        if (int rc = make_events(c)) {
            destroy_comms();
            return rc;
        }
    }
    g_mode = kCommLocal;
    g_nranks = n;
    return HEXCUDA_OK;
}

// Enqueues the gather of `nparts` row parts.  sends[p] / recvs[p] / streams[p]
// / comms[p] describe the parts this process drives (all of them in-process,
// one in a multi-process group: `first` is then its rank).
int enqueue_gather(int nparts, int first, int count, const void *const *sends, void *const *recvs,
                   const cudaStream_t *streams, const ncclComm_t *comms, int64_t rows,
                   size_t row_bytes) {
    std::vector<int64_t> r0((size_t)nparts + 1);
    for (int i = 0; i <= nparts; i++) r0[(size_t)i] = rows * i / nparts;
    bool equal = true;
    for (int i = 0; i < nparts; i++)
        equal = equal && (r0[(size_t)i + 1] - r0[(size_t)i]) == r0[1] - r0[0];
    if (int rc = ncheck(g_nccl.GroupStart(), "ncclGroupStart")) return rc;
    int rc = HEXCUDA_OK;
    for (int k = 0; k < count && !rc; k++) {
        const int me = first + k;
        uint8_t *recv = reinterpret_cast<uint8_t *>(recvs[k]);
        if (equal) {
            const size_t bytes = (size_t)(r0[1] - r0[0]) * row_bytes;
            rc = ncheck(g_nccl.AllGather(sends[k], recv, bytes, ncclUint8, comms[k], streams[k]),
                        "ncclAllGather");
            continue;
        }
        for (int root = 0; root < nparts && !rc; root++) {
            const size_t bytes = (size_t)(r0[(size_t)root + 1] - r0[(size_t)root]) * row_bytes;
            if (!bytes) continue;
            uint8_t *dst = recv + (size_t)r0[(size_t)root] * row_bytes;
            const void *src = root == me ? sends[k] : dst;
            rc = ncheck(g_nccl.Broadcast(src, dst, bytes, ncclUint8, root, comms[k], streams[k]),
                        "ncclBroadcast");
        }
    }
    const int rc2 = ncheck(g_nccl.GroupEnd(), "ncclGroupEnd");
    return rc ? rc : rc2;
}

int gather_local(const void *const *sends, void *const *recvs, int64_t rows, size_t row_bytes) {
    if (int rc = ensure_local_comms()) return rc;
    const int n = ndev();
    std::vector<cudaStream_t> streams((size_t)n);
    std::vector<ncclComm_t> comms((size_t)n);
    for (int i = 0; i < n; i++) {
        Dev *d = get_dev(i);
        if (!d) return hexcuda_last_error();
        streams[(size_t)i] = d->stream;
        comms[(size_t)i] = g_cd[(size_t)i].comm;
        if (int rc = check(cudaEventRecord(g_cd[(size_t)i].e0, d->stream), "event")) return rc;
    }
    if (int rc = enqueue_gather(n, 0, n, sends, recvs, streams.data(), comms.data(), rows,
                                row_bytes))
        return rc;
    for (int i = 0; i < n; i++) {
        Dev *d = get_dev(i);
        if (int rc = check(cudaEventRecord(g_cd[(size_t)i].e1, d->stream), "event")) return rc;
    }
    g_coll_ms = -2.0f;   // pending: read on demand
    return HEXCUDA_OK;
}

}  // namespace

bool replicate_on() { return g_replicate; }

// Called by the host entries after every part's output is enqueued: gathers
// the parts (device slot i's part at douts[i], null for an empty part) into
// each device's replica buffer.
int replicate_rows(const std::vector<void *> &douts, int64_t rows, size_t row_bytes) {
    if (!g_replicate) return HEXCUDA_OK;
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const int n = ndev();
    if ((int)douts.size() != n) return fail(HEXCUDA_ERR_ARG, "replicate: %d parts for %d devices",
                                            (int)douts.size(), n);
    if (int rc = ensure_local_comms()) return rc;
    const size_t bytes = (size_t)rows * row_bytes;
    std::vector<const void *> sends((size_t)n);
    std::vector<void *> recvs((size_t)n);
    for (int i = 0; i < n; i++) {
        Dev *d = get_dev(i);
        if (!d) return hexcuda_last_error();
        void *rep = scratch(d, kSlotReplica, bytes);
        if (!rep) return hexcuda_last_error();
        g_cd[(size_t)i].replica = rep;
        g_cd[(size_t)i].replica_bytes = bytes;
        recvs[(size_t)i] = rep;
        // an empty part sends nothing; any valid address will do
        sends[(size_t)i] = douts[(size_t)i] ? douts[(size_t)i] : rep;
    }
    return gather_local(sends.data(), recvs.data(), rows, row_bytes);
}

void replica_clear() {
    for (auto &c : g_cd) {
        c.replica = nullptr;
        c.replica_bytes = 0;
    }
}

void collective_release() { destroy_comms(); }

}  // namespace hx

using namespace hx;

HX_EXPORT int hexcuda_shard_rows(int64_t rows, int nparts, int part, int64_t *r0, int64_t *r1) {
    if (rows < 0 || nparts <= 0 || part < 0 || part >= nparts || !r0 || !r1)
        return fail(HEXCUDA_ERR_ARG, "shard_rows: rows=%lld nparts=%d part=%d", (long long)rows,
                    nparts, part);
    *r0 = rows * part / nparts;
    *r1 = rows * (part + 1) / nparts;
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_set_replicate(int on) {
    g_replicate = on != 0;
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_get_replicate(void) { return g_replicate ? 1 : 0; }

HX_EXPORT int hexcuda_replica(int dev, void **ptr, size_t *bytes) {
    if (!ptr || !bytes) return fail(HEXCUDA_ERR_ARG, "replica: null pointer");
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    if (g_mode != kCommLocal || dev < 0 || dev >= (int)g_cd.size() || !g_cd[(size_t)dev].replica)
        return fail(HEXCUDA_ERR_ARG, "replica: no replicated output on device slot %d", dev);
    *ptr = g_cd[(size_t)dev].replica;
    *bytes = g_cd[(size_t)dev].replica_bytes;
    return HEXCUDA_OK;
}

HX_EXPORT float hexcuda_last_collective_ms(void) {
    if (g_coll_ms != -2.0f) return g_coll_ms;
    float best = -1.0f;
    for (auto &c : g_cd) {
        if (!c.e1) continue;
        cudaSetDevice(c.ordinal);
        if (cudaEventSynchronize(c.e1) != cudaSuccess) continue;
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, c.e0, c.e1) == cudaSuccess && ms > best) best = ms;
    }
    g_coll_ms = best;
    return best;
}

HX_EXPORT int hexcuda_allgather_rows(const void *const *shards, void *const *fulls, int64_t rows,
                                     size_t row_bytes) {
    if (!shards || !fulls || rows < 0) return fail(HEXCUDA_ERR_ARG, "allgather_rows: bad arguments");
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    const int n = ndev();
    for (int i = 0; i < n; i++) {
        const bool empty = rows * (i + 1) / n == rows * i / n;
        if (!fulls[i] || (!shards[i] && !empty))
            return fail(HEXCUDA_ERR_ARG, "allgather_rows: null buffer for device slot %d", i);
    }
    if (rows == 0 || row_bytes == 0) return HEXCUDA_OK;
    std::vector<const void *> sends((size_t)n);
    for (int i = 0; i < n; i++) sends[(size_t)i] = shards[i] ? shards[i] : fulls[i];
    return gather_local(sends.data(), fulls, rows, row_bytes);
}

HX_EXPORT int hexcuda_comm_unique_id(void *id, size_t id_bytes) {
    if (!id || id_bytes < sizeof(ncclUniqueId))
        return fail(HEXCUDA_ERR_ARG, "comm_unique_id: need %zu bytes", sizeof(ncclUniqueId));
    if (!nccl_load()) return hexcuda_last_error();
    ncclUniqueId u;
    if (int rc = ncheck(g_nccl.GetUniqueId(&u), "ncclGetUniqueId")) return rc;
    memcpy(id, &u, sizeof(u));
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_comm_init_rank(int nranks, int rank, const void *id, size_t id_bytes) {
    if (nranks <= 0 || rank < 0 || rank >= nranks || !id || id_bytes < sizeof(ncclUniqueId))
        return fail(HEXCUDA_ERR_ARG, "comm_init_rank: nranks=%d rank=%d", nranks, rank);
    if (!ensure_init()) return HEXCUDA_ERR_NODEV;
    if (ndev() != 1)
        return fail(HEXCUDA_ERR_ARG,
                    "comm_init_rank: one device per process expected (%d initialised)", ndev());
    if (!nccl_load()) return hexcuda_last_error();
    destroy_comms();
    Dev *d = get_dev(0);
    if (!d) return hexcuda_last_error();
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t comm = nullptr;
    if (int rc = ncheck(g_nccl.CommInitRank(&comm, nranks, u, rank), "ncclCommInitRank")) return rc;
    g_cd.assign(1, CollDev());
    g_cd[0].ordinal = d->ordinal;
    g_cd[0].comm = comm;
    if (int rc = make_events(g_cd[0])) {
        destroy_comms();
        return rc;
    }
    g_mode = kCommRank;
    g_nranks = nranks;
    g_rank = rank;
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_comm_destroy(void) {
    destroy_comms();
    return HEXCUDA_OK;
}

HX_EXPORT int hexcuda_comm_allgather_rows(const void *shard, void *full, int64_t rows,
                                          size_t row_bytes) {
    if (g_mode != kCommRank)
        return fail(HEXCUDA_ERR_ARG, "comm_allgather_rows: no multi-process group "
                                     "(call hexcuda_comm_init_rank first)");
    if (!full || rows < 0) return fail(HEXCUDA_ERR_ARG, "comm_allgather_rows: bad arguments");
    const bool empty = rows * (g_rank + 1) / g_nranks == rows * g_rank / g_nranks;
    if (!shard && !empty) return fail(HEXCUDA_ERR_ARG, "comm_allgather_rows: null shard");
    if (rows == 0 || row_bytes == 0) return HEXCUDA_OK;
    Dev *d = get_dev(0);
    if (!d) return hexcuda_last_error();
    CollDev &c = g_cd[0];
    const void *send = shard ? shard : full;
    if (int rc = check(cudaEventRecord(c.e0, d->stream), "event")) return rc;
    if (int rc = enqueue_gather(g_nranks, g_rank, 1, &send, &full, &d->stream, &c.comm, rows,
                                row_bytes))
        return rc;
    if (int rc = check(cudaEventRecord(c.e1, d->stream), "event")) return rc;
    g_coll_ms = -2.0f;
    return HEXCUDA_OK;
}
