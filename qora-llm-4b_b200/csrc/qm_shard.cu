// Multi-GPU support: the head-sharded layout of the decode stack and the one
// collective it needs, an all-gather of the mixer outputs.
//
// The reference runs on one device (src/gpu_inference.rs:981-1004); its
// batch is one sequence.  Here sequences shard across GPUs with no
// communication at all (each rank owns whole states and caches), and a
// second layout shards the heads of every layer:
//   DeltaNet  V heads [r*32/N, (r+1)*32/N); V heads 2j and 2j+1 share QK
//             head j (src/gemv.rs:803-809), so N <= 16 keeps each QK head's
//             conv history on one rank;
//   GQA       min(N,4) groups of 4/min(N,4) KV heads; with N > 4 ranks the
//             batch splits into N/4 equal parts on top.
// Each rank then holds 1/N of every state and cache and the per-layer mixer
// output must be gathered before out_proj / o_proj.  That all-gather is the
// only data exchanged; NCCL is loaded at run time (libnccl.so.2: the copy a
// host process such as PyTorch already loaded, else the system one), so the
// library has no link-time NCCL dependency.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>

#include "qm_internal.h"

using namespace qm;

extern "C" int qm_shard_plan(int world, int rank, qm_shard* out) {
    if (!out || world < 1 || rank < 0 || rank >= world) return QM_E_ARG;
    if (world > 16 || (kNumV % world) != 0) return QM_E_SHAPE;  // 1, 2, 4, 8, 16
    const int groups = world < kNumKVH ? world : kNumKVH;
    if ((kNumKVH % groups) != 0 || (world % groups) != 0) return QM_E_SHAPE;
    out->world = world;
    out->rank = rank;
    out->nvh = kNumV / world;
    out->vh_lo = rank * out->nvh;
    out->nkv = kNumKVH / groups;
    out->kv_lo = (rank % groups) * out->nkv;
    out->seq_parts = world / groups;
    out->seq_part = rank / groups;
    return QM_OK;
}

// ---------------------------------------------------------------------------
// NCCL, resolved with dlsym
// ---------------------------------------------------------------------------
namespace {

struct NcclApi {
    bool tried = false, ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

const NcclApi* nccl_api() {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.tried) return &g_nccl;
    g_nccl.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        g_nccl.why = std::string("libnccl.so.2 not loadable: ") + dlerror();
        return &g_nccl;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(sym("ncclGetUniqueId"));
    g_nccl.init_rank_config =
        reinterpret_cast<decltype(g_nccl.init_rank_config)>(sym("ncclCommInitRankConfig"));
    g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(sym("ncclAllGather"));
    g_nccl.async_error = reinterpret_cast<decltype(g_nccl.async_error)>(sym("ncclCommGetAsyncError"));
    g_nccl.finalize = reinterpret_cast<decltype(g_nccl.finalize)>(sym("ncclCommFinalize"));
    g_nccl.destroy = reinterpret_cast<decltype(g_nccl.destroy)>(sym("ncclCommDestroy"));
    g_nccl.abort = reinterpret_cast<decltype(g_nccl.abort)>(sym("ncclCommAbort"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(sym("ncclGetErrorString"));
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.init_rank_config && g_nccl.all_gather &&
                g_nccl.async_error && g_nccl.finalize && g_nccl.destroy && g_nccl.abort &&
                g_nccl.error_string;
    if (!g_nccl.ok) g_nccl.why = "libnccl.so.2 lacks a required symbol";
    return &g_nccl;
}

}  // namespace

struct qm_comm {
    qm_ctx* ctx = nullptr;    // for calls; destroy uses `device` only (ctx may be gone)
    int device = 0;
    ncclComm_t comm = nullptr;
    int world = 0, rank = 0;
    int timeout_ms = 0;
};

// Non-blocking communicator: every call may return ncclInProgress; poll the
// async error with a time limit and abort the communicator past it.
// Returns the final NCCL result (ncclInProgress = timed out and aborted).
static ncclResult_t nccl_poll(qm_comm* c, ncclResult_t r) {
    const NcclApi* api = nccl_api();
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms)) {
            api->abort(c->comm);
            c->comm = nullptr;
            return ncclInProgress;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
        if (api->async_error(c->comm, &r) != ncclSuccess) break;
    }
    return r;
}

static int nccl_wait(qm_comm* c, ncclResult_t r, const char* what) {
    r = nccl_poll(c, r);
    if (r == ncclInProgress)
        return set_error(c->ctx, QM_E_TIMEOUT, std::string(what) + ": NCCL did not complete in time");
    if (r != ncclSuccess)
        return set_error(c->ctx, QM_E_NCCL, std::string(what) + ": " + nccl_api()->error_string(r));
    return QM_OK;
}

extern "C" int qm_comm_unique_id(unsigned char* id) {
    if (!id) return QM_E_ARG;
    static_assert(sizeof(ncclUniqueId) == QM_COMM_ID_BYTES, "NCCL unique id size");
    const NcclApi* api = nccl_api();
    if (!api->ok) return QM_E_NCCL;
    ncclUniqueId u;
    if (api->get_unique_id(&u) != ncclSuccess) return QM_E_NCCL;
    memcpy(id, &u, sizeof(u));
    return QM_OK;
}

extern "C" int qm_comm_create(qm_ctx* ctx, const unsigned char* id, int world, int rank,
                              int timeout_ms, qm_comm** out) {
    if (!ctx) return QM_E_ARG;
    if (!id || !out || world < 1 || rank < 0 || rank >= world || timeout_ms <= 0)
        return set_error(ctx, QM_E_ARG, "qm_comm_create: bad argument");
    *out = nullptr;
    const NcclApi* api = nccl_api();
    if (!api->ok) return set_error(ctx, QM_E_NCCL, api->why);
    qm_comm* c = new (std::nothrow) qm_comm();
    if (!c) return QM_E_OOM;
    c->ctx = ctx;
    c->device = ctx->device;
    c->world = world;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    cudaSetDevice(ctx->device);
    int rc = nccl_wait(c, api->init_rank_config(&c->comm, world, u, rank, &cfg), "ncclCommInitRank");
    if (rc != QM_OK) {
        if (c->comm) api->abort(c->comm);
        delete c;
        return rc;
    }
    *out = c;
    return QM_OK;
}

extern "C" int qm_comm_allgather(qm_comm* c, const void* send, void* recv, size_t bytes_per_rank) {
    if (!c) return QM_E_ARG;
    if (!c->comm) return set_error(c->ctx, QM_E_NCCL, "communicator was aborted");
    if (!send || !recv || bytes_per_rank == 0)
        return set_error(c->ctx, QM_E_ARG, "qm_comm_allgather: bad argument");
    const NcclApi* api = nccl_api();
    cudaSetDevice(c->ctx->device);
    TimedLaunch tl(c->ctx, "allgather");
    return nccl_wait(c, api->all_gather(send, recv, bytes_per_rank, ncclUint8, c->comm, c->ctx->stream),
                     "ncclAllGather");
}

extern "C" int qm_comm_destroy(qm_comm* c) {
    if (!c) return QM_E_ARG;
    if (c->comm) {
        const NcclApi* api = nccl_api();
        cudaSetDevice(c->device);
        // non-blocking communicator: finalize (flushes outstanding work), then free
        const ncclResult_t r = nccl_poll(c, api->finalize(c->comm));
        if (r == ncclSuccess)
            api->destroy(c->comm);
        else if (c->comm)
            api->abort(c->comm);
    }
    delete c;
    return QM_OK;
}
