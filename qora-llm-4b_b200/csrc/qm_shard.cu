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
// only data exchanged.  It runs through NCCL, loaded at run time
// (libnccl.so.2: the copy a host process such as PyTorch already loaded,
// else the system one, so the library has no link-time NCCL dependency), or,
// after qm_comm_enable_peer, through this file's peer-memory kernel.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

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

namespace {

// ---------------------------------------------------------------------------
// Peer-memory all-gather (qm_comm_enable_peer)
// ---------------------------------------------------------------------------
// Every rank cudaMalloc's one gather area, exports it (cudaIpcGetMemHandle)
// and maps every other rank's (handles exchanged over the communicator):
//   flags [2 slots][world][kPeerChunks] u32   epoch of the last write
//   data  [2 slots][world][max_bytes]         row = source rank
// A call with epoch e uses slot e & 1.  Block (j, c) of the gather kernel
// stores chunk c of this rank's send into rank j's area, row `rank`, with
// plain stores through the peer mapping (NVLink), publishes it with a
// system-scope release store of flags[slot][rank][c] = e on rank j, then
// waits (bounded) until rank j's flag for chunk c in this rank's own area
// reads e and copies that chunk into recv.  Block (rank, c) copies send
// straight into recv.  Slot reuse is safe: rank j writes slot s again only
// at epoch e + 2, after its call e + 1 finished; that call needed this
// rank's call-(e + 1) flag, written after this rank's call e (same stream)
// had copied slot s out.
constexpr int kPeerMaxWorld = 16;
constexpr int kPeerChunks = 64;
constexpr size_t kPeerChunkMin = 4096;
constexpr size_t kPeerDataOff = 2 * kPeerMaxWorld * kPeerChunks * sizeof(unsigned);  // 8 KB
constexpr int kPeerThreads = 512;

struct PeerGatherArgs {
    const unsigned char* send;
    unsigned char* recv;
    unsigned char* area[kPeerMaxWorld];  // every rank's gather area as mapped here
    size_t bytes;                        // per rank
    size_t max_bytes;                    // row pitch of the data slots (multiple of 16)
    size_t chunk;                        // bytes per chunk (multiple of 16)
    int world, rank, chunks, slot, vec;
    unsigned epoch;
    unsigned long long wait_ns;
    int* err;                            // context error word
    int* fail;                           // host-mapped failure word of the communicator
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned* peer_flag(unsigned char* area, int world, int slot, int src,
                                               int c) {
    return reinterpret_cast<unsigned*>(area) + ((size_t)slot * world + src) * kPeerChunks + c;
}

// Copies [lo, hi) of src to dst (16-byte vectors when every address and the
// per-rank size are 16-byte multiples, bytes otherwise).  `cg` reads with
// ld.global.cg (L2 only): the data was written by another GPU.
__device__ __forceinline__ void block_copy(unsigned char* dst, const unsigned char* src, size_t n,
                                           bool vec, bool cg) {
    if (vec) {
        uint4* d = reinterpret_cast<uint4*>(dst);
        const uint4* s = reinterpret_cast<const uint4*>(src);
        for (size_t i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = cg ? __ldcg(s + i) : s[i];
    } else {
        for (size_t i = threadIdx.x; i < n; i += blockDim.x)
            dst[i] = cg ? (unsigned char)__ldcg(reinterpret_cast<const char*>(src) + i) : src[i];
    }
}

__global__ void __launch_bounds__(kPeerThreads) peer_allgather_kernel(PeerGatherArgs a) {
    const int j = blockIdx.x / a.chunks;
    const int c = blockIdx.x % a.chunks;
    const size_t lo = (size_t)c * a.chunk;
    if (lo >= a.bytes) return;
    const size_t n = (a.bytes - lo < a.chunk) ? a.bytes - lo : a.chunk;
    const bool vec = a.vec != 0;
    if (j == a.rank) {
        block_copy(a.recv + (size_t)a.rank * a.bytes + lo, a.send + lo, n, vec, false);
        return;
    }
    // push: this rank's chunk into rank j's area, then the flag
    unsigned char* row =
        a.area[j] + kPeerDataOff + ((size_t)a.slot * a.world + a.rank) * a.max_bytes;
    block_copy(row + lo, a.send + lo, n, vec, false);
    __syncthreads();
    __shared__ int ok;
    if (threadIdx.x == 0) {
        // the barrier orders the block's stores before this thread's
        // system-scope fence, which the release store then publishes
        __threadfence_system();
        st_release_sys(peer_flag(a.area[j], a.world, a.slot, a.rank, c), a.epoch);
        // wait (bounded) for rank j's chunk c in this rank's own area
        const unsigned* f = peer_flag(a.area[a.rank], a.world, a.slot, j, c);
        const unsigned long long t0 = global_ns();
        int good = 1;
        while (ld_acquire_sys(f) != a.epoch) {
            if (global_ns() - t0 > a.wait_ns) {
                good = 0;
                atomicOr(a.err, kErrTimeout);
                *reinterpret_cast<volatile int*>(a.fail) = 1;
                break;
            }
        }
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    const unsigned char* src =
        a.area[a.rank] + kPeerDataOff + ((size_t)a.slot * a.world + j) * a.max_bytes;
    block_copy(a.recv + (size_t)j * a.bytes + lo, src + lo, n, vec, true);
}

struct PeerRec {              // what each rank publishes at qm_comm_enable_peer
    cudaIpcMemHandle_t handle;
    unsigned char uuid[16];
    int ok;
    int pad;
};

}  // namespace

struct qm_comm {
    qm_ctx* ctx = nullptr;    // for calls; destroy uses `device` only (ctx may be gone)
    int device = 0;
    ncclComm_t comm = nullptr;
    int world = 0, rank = 0;
    int timeout_ms = 0;
    // peer-memory all-gather (qm_comm_enable_peer)
    bool peer = false;
    unsigned char* area[kPeerMaxWorld] = {};  // own at [rank]; others are IPC mappings
    size_t peer_max = 0;
    unsigned long long wait_ns = 0;
    unsigned epoch = 0;
    int* fail_h = nullptr;                    // host-mapped failure word
    int* fail_d = nullptr;
    cudaStream_t side = nullptr;              // set-up / tear-down collectives
    void* scratch = nullptr;                  // device bytes for those collectives
    cudaEvent_t done = nullptr;               // after the last gather kernel
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

// Waits (bounded by the communicator's timeout) for the side stream; past
// the limit the communicator is aborted, which ends NCCL's kernel.
static bool side_wait(qm_comm* c) {
    cudaEvent_t ev = nullptr;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return false;
    cudaEventRecord(ev, c->side);
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e;
    while ((e = cudaEventQuery(ev)) == cudaErrorNotReady) {
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms)) {
            if (c->comm) nccl_api()->abort(c->comm);
            c->comm = nullptr;
            cudaEventDestroy(ev);
            return false;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    cudaEventDestroy(ev);
    return e == cudaSuccess;
}

// One all-gather of `bytes` host bytes per rank through c->scratch on the
// side stream (set-up and tear-down of the peer path only).
static bool side_allgather(qm_comm* c, const void* mine, void* all, size_t bytes) {
    if (!c->comm) return false;
    unsigned char* d = static_cast<unsigned char*>(c->scratch);
    if (cudaMemcpyAsync(d, mine, bytes, cudaMemcpyHostToDevice, c->side) != cudaSuccess) return false;
    if (nccl_poll(c, nccl_api()->all_gather(d, d + bytes, bytes, ncclUint8, c->comm, c->side)) !=
        ncclSuccess)
        return false;
    if (cudaMemcpyAsync(all, d + bytes, bytes * c->world, cudaMemcpyDeviceToHost, c->side) !=
        cudaSuccess)
        return false;
    return side_wait(c);
}

// Undoes qm_comm_enable_peer.  The own area is freed only after every rank
// has unmapped it (an all-gather after the unmapping); when that cannot be
// shown (aborted communicator) the area is left allocated.
static void peer_release(qm_comm* c) {
    cudaSetDevice(c->device);
    if (c->done) cudaEventSynchronize(c->done);  // the last gather kernel (bounded waits)
    for (int j = 0; j < c->world; j++)
        if (j != c->rank && c->area[j]) cudaIpcCloseMemHandle(c->area[j]);
    int one = 1;
    std::vector<int> all(c->world);
    const bool unmapped_everywhere = c->side && c->scratch && side_allgather(c, &one, all.data(), sizeof(int));
    if (unmapped_everywhere) {
        cudaFree(c->area[c->rank]);
        cudaFree(c->scratch);
    }
    if (c->fail_h) cudaFreeHost(c->fail_h);
    if (c->done) cudaEventDestroy(c->done);
    if (c->side) cudaStreamDestroy(c->side);
    for (int j = 0; j < kPeerMaxWorld; j++) c->area[j] = nullptr;
    c->fail_h = c->fail_d = nullptr;
    c->scratch = nullptr;
    c->side = nullptr;
    c->done = nullptr;
    c->peer = false;
}

extern "C" int qm_comm_enable_peer(qm_comm* c, size_t max_bytes_per_rank, int wait_ms) {
    if (!c) return QM_E_ARG;
    if (!c->comm) return set_error(c->ctx, QM_E_NCCL, "communicator was aborted");
    if (max_bytes_per_rank == 0 || wait_ms <= 0)
        return set_error(c->ctx, QM_E_ARG, "qm_comm_enable_peer: bad argument");
    if (c->peer) return set_error(c->ctx, QM_E_ARG, "qm_comm_enable_peer: already enabled");
    if (c->world > kPeerMaxWorld)
        return set_error(c->ctx, QM_E_UNSUPPORTED, "qm_comm_enable_peer: more than 16 ranks");
    cudaSetDevice(c->device);
    // the side stream and scratch carry the set-up collectives; without them
    // this rank cannot take part (the others' exchange then times out)
    if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->scratch, (size_t)(c->world + 1) * sizeof(PeerRec)) != cudaSuccess) {
        cudaGetLastError();
        peer_release(c);
        return set_error(c->ctx, QM_E_OOM, "qm_comm_enable_peer: set-up stream / scratch");
    }
    // every later failure still takes part in both exchanges, with ok = 0
    const size_t maxb = (max_bytes_per_rank + 15) / 16 * 16;
    unsigned char* own = nullptr;
    bool setup = cudaMalloc(&own, kPeerDataOff + 2 * (size_t)c->world * maxb) == cudaSuccess;
    if (setup) c->area[c->rank] = own;
    // flags zeroed on the side stream, ahead of the exchanges that publish them
    setup = setup && cudaMemsetAsync(own, 0, kPeerDataOff, c->side) == cudaSuccess &&
            cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming) == cudaSuccess &&
            cudaHostAlloc(reinterpret_cast<void**>(&c->fail_h), sizeof(int), cudaHostAllocMapped) ==
                cudaSuccess;
    if (setup) {
        *c->fail_h = 0;
        setup = cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->fail_d), c->fail_h, 0) == cudaSuccess;
    }
    PeerRec mine{};
    mine.ok = setup && (c->world == 1 || cudaIpcGetMemHandle(&mine.handle, own) == cudaSuccess);
    cudaDeviceProp prop;
    if (mine.ok && cudaGetDeviceProperties(&prop, c->device) == cudaSuccess)
        memcpy(mine.uuid, prop.uuid.bytes, sizeof(mine.uuid));
    else
        mine.ok = 0;
    cudaGetLastError();
    std::vector<PeerRec> recs(c->world);
    if (!side_allgather(c, &mine, recs.data(), sizeof(PeerRec))) {
        peer_release(c);
        return set_error(c->ctx, QM_E_TIMEOUT, "qm_comm_enable_peer: exchanging the gather areas failed");
    }
    int ok = mine.ok;
    for (int j = 0; j < c->world && ok; j++) {
        if (j == c->rank) continue;
        // two ranks on one GPU would wait on each other inside one device: refuse
        if (!recs[j].ok || memcmp(recs[j].uuid, mine.uuid, sizeof(mine.uuid)) == 0) {
            ok = 0;
            break;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, recs[j].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
            break;
        }
        c->area[j] = static_cast<unsigned char*>(p);
    }
    std::vector<int> oks(c->world);
    bool all_ok = side_allgather(c, &ok, oks.data(), sizeof(int));
    for (int j = 0; j < c->world && all_ok; j++) all_ok = oks[j] != 0;
    if (!all_ok) {
        const bool aborted = c->comm == nullptr;
        peer_release(c);
        return set_error(c->ctx, aborted ? QM_E_TIMEOUT : QM_E_UNSUPPORTED,
                         "qm_comm_enable_peer: a rank cannot map every other rank's memory "
                         "(or two ranks share a GPU); the NCCL all-gather stays in use");
    }
    c->peer = true;
    c->peer_max = maxb;
    c->wait_ns = (unsigned long long)wait_ms * 1000000ull;
    c->epoch = 0;
    return QM_OK;
}

static int peer_allgather(qm_comm* c, const void* send, void* recv, size_t bytes) {
    if (*reinterpret_cast<volatile int*>(c->fail_h))
        return set_error(c->ctx, QM_E_TIMEOUT,
                         "peer all-gather: a wait of an earlier call gave up, the ranks are out of "
                         "step; destroy the communicator");
    PeerGatherArgs a{};
    a.send = static_cast<const unsigned char*>(send);
    a.recv = static_cast<unsigned char*>(recv);
    for (int j = 0; j < c->world; j++) a.area[j] = c->area[j];
    a.bytes = bytes;
    a.max_bytes = c->peer_max;
    size_t chunks = bytes / kPeerChunkMin;
    chunks = chunks < 1 ? 1 : (chunks > (size_t)kPeerChunks ? kPeerChunks : chunks);
    a.chunk = ((bytes + chunks - 1) / chunks + 15) / 16 * 16;
    a.chunks = (int)chunks;
    a.world = c->world;
    a.rank = c->rank;
    a.epoch = ++c->epoch;
    a.slot = (int)(a.epoch & 1u);
    a.vec = ((reinterpret_cast<uintptr_t>(send) | reinterpret_cast<uintptr_t>(recv) | bytes) & 15) == 0;
    a.wait_ns = c->wait_ns;
    a.err = c->ctx->d_err;
    a.fail = c->fail_d;
    TimedLaunch tl(c->ctx, "allgather");
    peer_allgather_kernel<<<c->world * a.chunks, kPeerThreads, 0, c->ctx->stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(c->ctx, e, "peer_allgather_kernel");
    c->ctx->launches += 1;
    cudaEventRecord(c->done, c->ctx->stream);
    return QM_OK;
}

extern "C" int qm_comm_allgather(qm_comm* c, const void* send, void* recv, size_t bytes_per_rank) {
    if (!c) return QM_E_ARG;
    if (!c->comm) return set_error(c->ctx, QM_E_NCCL, "communicator was aborted");
    if (!send || !recv || bytes_per_rank == 0)
        return set_error(c->ctx, QM_E_ARG, "qm_comm_allgather: bad argument");
    cudaSetDevice(c->device);
    if (c->peer && bytes_per_rank <= c->peer_max) return peer_allgather(c, send, recv, bytes_per_rank);
    const NcclApi* api = nccl_api();
    TimedLaunch tl(c->ctx, "allgather");
    return nccl_wait(c, api->all_gather(send, recv, bytes_per_rank, ncclUint8, c->comm, c->ctx->stream),
                     "ncclAllGather");
}

extern "C" int qm_comm_destroy(qm_comm* c) {
    if (!c) return QM_E_ARG;
    if (c->peer) peer_release(c);
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
