// C-ABI front end: contexts, state/cache handles, argument checks, _host
// variants.  Kernels live in dn_decode.cu, gqa_decode.cu, gqa_prefill.cu and
// dn_prefill.cu.
#include <cudaTypedefs.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <new>
#include <vector>

#include "qm_internal.h"

using namespace qm;

namespace qm {

int set_error(qm_ctx* ctx, int code, const std::string& msg) {
    if (ctx) ctx->last_error = msg;
    return code;
}

int cuda_error(qm_ctx* ctx, cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return set_error(ctx, QM_E_OOM, m);
    return set_error(ctx, QM_E_CUDA, m);
}

static bool stream_capturing(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &st) != cudaSuccess) return false;
    return st != cudaStreamCaptureStatusNone;
}

int ensure_workspace(qm_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->ws_bytes) return QM_OK;
    if (stream_capturing(ctx->stream))
        return set_error(ctx, QM_E_CAPTURE,
                         "workspace must grow during stream capture; call qm_ctx_reserve first");
    QM_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->ws) cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    size_t want = (bytes + 0xFFFFF) & ~size_t(0xFFFFF);
    QM_CHECK_CUDA(ctx, cudaMalloc(&ctx->ws, want));
    ctx->ws_bytes = want;
    return QM_OK;
}

int ensure_stage(qm_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->stage_bytes) return QM_OK;
    if (stream_capturing(ctx->stream))
        return set_error(ctx, QM_E_CAPTURE, "staging buffer must grow during stream capture");
    QM_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->stage) cudaFree(ctx->stage);
    ctx->stage = nullptr;
    ctx->stage_bytes = 0;
    size_t want = (bytes + 0xFFFFF) & ~size_t(0xFFFFF);
    QM_CHECK_CUDA(ctx, cudaMalloc(&ctx->stage, want));
    ctx->stage_bytes = want;
    return QM_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_tiled() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// cuPointerGetAttributes, resolved once through the runtime (no link-time
// libcuda dependency).
typedef CUresult (*PFN_pointer_get_attributes)(unsigned int, CUpointer_attribute*, void**, CUdeviceptr);
static PFN_pointer_get_attributes get_pointer_attributes() {
    static PFN_pointer_get_attributes fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuPointerGetAttributes", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_pointer_get_attributes>(p);
    });
    return fn;
}

// The device address of host bytes [p, p + bytes) when the kernels can use
// them in place: page-locked host memory, mapped into the current device's
// address space, with the whole range inside one allocation.  Anything else
// (pageable memory, a range that runs past its allocation, a failed query)
// gives nullptr and the caller stages the bytes through copies.
static void* mapped_host(const void* p, size_t bytes) {
    PFN_pointer_get_attributes get = get_pointer_attributes();
    if (!get || !p) return nullptr;
    unsigned int mtype = 0;
    CUdeviceptr start = 0, dptr = 0;
    size_t size = 0;
    CUpointer_attribute attrs[4] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                    CU_POINTER_ATTRIBUTE_RANGE_SIZE, CU_POINTER_ATTRIBUTE_DEVICE_POINTER};
    void* data[4] = {&mtype, &start, &size, &dptr};
    // (unknown pointers give CUDA_SUCCESS with zeroed attributes)
    if (get(4, attrs, data, (CUdeviceptr)p) != CUDA_SUCCESS) return nullptr;
    if (mtype != CU_MEMORYTYPE_HOST || !dptr || !size) return nullptr;
    const uintptr_t a = (uintptr_t)p;
    if (a < (uintptr_t)start || bytes > size || a - (uintptr_t)start > size - bytes) return nullptr;
    return reinterpret_cast<void*>(dptr);
}

// Ends an in-place host call: the error word follows the kernels on the
// context stream, one synchronisation covers the kernels' host writes too.
static int direct_finish(qm_ctx* c) {
    QM_CHECK_CUDA(c, cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->stream));
    const int err = *c->h_err;
    if (err) {
        cudaMemset(c->d_err, 0, sizeof(int));
        if (err & kErrBounds)
            return set_error(c, QM_E_RANGE, "a device-side index self-check failed (access skipped)");
        return set_error(c, QM_E_TIMEOUT, "a device-side bounded wait gave up (error word set)");
    }
    return QM_OK;
}

extern "C" int qm_ctx_set_host_direct(qm_ctx* c, int on) {
    if (!c) return QM_E_ARG;
    c->host_direct = on != 0;
    return QM_OK;
}

extern "C" int qm_ctx_host_calls(const qm_ctx* c, int64_t* in_place, int64_t* staged) {
    if (!c) return QM_E_ARG;
    if (in_place) *in_place = c->host_in_place;
    if (staged) *staged = c->host_staged;
    return QM_OK;
}

// 3-D bf16 view of a cache [planes = B*nkv][cap][256]: box {64 dims, 64
// positions, 1}, 128-byte swizzle, zero fill past the capacity.
int encode_cache_tmap(CUtensorMap* m, void* base, int planes, int capacity, int box_rows) {
    auto enc = get_encode_tiled();
    if (!enc) return QM_E_CUDA;
    cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)capacity, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)capacity * kD * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? QM_OK : QM_E_CUDA;
}

// Generic 3-D bf16 view {inner, rows, planes} (row-major), 128-byte swizzle.
int encode_rows_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                     uint32_t box_inner, uint32_t box_rows, bool fp16) {
    auto enc = get_encode_tiled();
    if (!enc) return QM_E_CUDA;
    cuuint64_t dims[3] = {inner, rows, planes};
    cuuint64_t strides[2] = {inner * 2, rows * inner * 2};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                     base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? QM_OK : QM_E_CUDA;
}

// 3-D f32 view {inner, rows, planes} (row-major), no swizzle: the plain
// row-major tiles a TMA store writes from shared memory (out-of-range rows
// are skipped).
int encode_f32_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                    uint32_t box_inner, uint32_t box_rows) {
    auto enc = get_encode_tiled();
    if (!enc) return QM_E_CUDA;
    cuuint64_t dims[3] = {inner, rows, planes};
    cuuint64_t strides[2] = {inner * 4, rows * inner * 4};
    cuuint32_t box[3] = {box_inner, box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? QM_OK : QM_E_CUDA;
}

int make_kv_tmaps(qm_kv* kv) {
    kv->tmaps_ok = false;
    const int planes = kv->batch * kv->nkv;
    if (encode_cache_tmap(&kv->tmap_k, kv->k, planes, kv->capacity, 64) != QM_OK ||
        encode_cache_tmap(&kv->tmap_v, kv->v, planes, kv->capacity, 64) != QM_OK)
        return set_error(kv->ctx, QM_E_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
    kv->tmaps_ok = true;
    return QM_OK;
}

}  // namespace qm

// ---------------------------------------------------------------------------
// status / shape
// ---------------------------------------------------------------------------
extern "C" int qm_build_flags(void) {
#ifdef QM_CHECK_BOUNDS
    return QM_BUILD_BOUNDS_CHECKS;
#else
    return 0;
#endif
}

extern "C" int qm_shape_get(qm_shape* o) {
    if (!o) return QM_E_ARG;
    o->num_qk_heads = kNumQK;
    o->num_v_heads = kNumV;
    o->dn_head_dim = kHd;
    o->conv_kernel = kConvK;
    o->num_attn_heads = kNumH;
    o->num_kv_heads = kNumKVH;
    o->attn_head_dim = kD;
    o->rope_dim = kRot;
    o->rope_theta = 1.0e7f;
    o->rms_eps = 1e-6f;
    return QM_OK;
}

extern "C" const char* qm_status_string(int s) {
    switch (s) {
        case QM_OK: return "ok";
        case QM_E_ARG: return "invalid argument";
        case QM_E_SHAPE: return "shape or capacity mismatch";
        case QM_E_OOM: return "out of device memory";
        case QM_E_CUDA: return "CUDA error";
        case QM_E_NCCL: return "NCCL error";
        case QM_E_TIMEOUT: return "device-side wait timed out";
        case QM_E_RANGE: return "position out of range";
        case QM_E_MISMATCH: return "handle mismatch";
        case QM_E_UNSUPPORTED: return "unsupported device";
        case QM_E_CAPTURE: return "allocation needed during stream capture";
        default: return "unknown status";
    }
}

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
static void drop_events(qm_ctx* c);
extern "C" int qm_ctx_create(int device, qm_ctx** out) {
    if (!out) return QM_E_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return QM_E_ARG;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return QM_E_CUDA;
    if (prop.major != 10) return QM_E_UNSUPPORTED;
    qm_ctx* c = new (std::nothrow) qm_ctx();
    if (!c) return QM_E_OOM;
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return QM_E_CUDA;
    }
    c->stream = c->own_stream;
    if (cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess ||
        cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess) {
        cudaStreamDestroy(c->own_stream);
        delete c;
        return QM_E_OOM;
    }
    *out = c;
    return QM_OK;
}

extern "C" int qm_ctx_destroy(qm_ctx* c) {
    if (!c) return QM_E_ARG;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->ws) cudaFree(c->ws);
    if (c->stage) cudaFree(c->stage);
    if (c->d_err) cudaFree(c->d_err);
    if (c->gemv_partial) cudaFree(c->gemv_partial);
    if (c->gemv_count) cudaFree(c->gemv_count);
    drop_events(c);
    for (cudaEvent_t e : c->event_pool) cudaEventDestroy(e);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    if (c->pipe_ready) {
        cudaStreamSynchronize(c->copy_in);
        cudaStreamSynchronize(c->copy_out);
        cudaStreamDestroy(c->copy_in);
        cudaStreamDestroy(c->copy_out);
        for (int i = 0; i < 8; i++) {
            cudaEventDestroy(c->pipe_in[i]);
            cudaEventDestroy(c->pipe_done[i]);
        }
        cudaFreeHost(c->h_err);
    }
    delete c;
    return QM_OK;
}

extern "C" int qm_ctx_set_stream(qm_ctx* c, void* stream) {
    if (!c) return QM_E_ARG;
    c->stream = (cudaStream_t)stream;  // taken verbatim: NULL is the legacy default stream
    return QM_OK;
}

extern "C" void* qm_ctx_get_stream(const qm_ctx* c) { return c ? (void*)c->stream : nullptr; }

extern "C" int qm_sync(qm_ctx* c) {
    if (!c) return QM_E_ARG;
    cudaSetDevice(c->device);
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->stream));
    int err = 0;
    QM_CHECK_CUDA(c, cudaMemcpy(&err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        cudaMemset(c->d_err, 0, sizeof(int));
        if (err & kErrBounds)
            return set_error(c, QM_E_RANGE, "a device-side index self-check failed (access skipped)");
        return set_error(c, QM_E_TIMEOUT, "a device-side bounded wait gave up (error word set)");
    }
    return QM_OK;
}

extern "C" const char* qm_last_error(const qm_ctx* c) {
    return c ? c->last_error.c_str() : "null context";
}

extern "C" int qm_ctx_reserve(qm_ctx* c, size_t bytes) {
    if (!c) return QM_E_ARG;
    cudaSetDevice(c->device);
    return ensure_workspace(c, bytes);
}

extern "C" int64_t qm_ctx_launch_count(const qm_ctx* c) { return c ? c->launches : -1; }

namespace qm {
static cudaEvent_t pool_event(qm_ctx* c) {
    if (!c->event_pool.empty()) {
        cudaEvent_t e = c->event_pool.back();
        c->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

TimedLaunch::TimedLaunch(qm_ctx* c, const char* name) : ctx(c) {
    if (!c->timing) return;
    cudaEvent_t start = pool_event(c);
    stop = pool_event(c);
    cudaEventRecord(start, c->stream);
    c->events[name].push_back({start, stop});
}

TimedLaunch::~TimedLaunch() {
    if (stop) cudaEventRecord(stop, ctx->stream);
}
}  // namespace qm

static void drop_events(qm_ctx* c) {
    for (auto& kv : c->events)
        for (auto& pr : kv.second) {
            c->event_pool.push_back(pr.first);
            c->event_pool.push_back(pr.second);
        }
    c->events.clear();
}

extern "C" int qm_ctx_set_timing(qm_ctx* c, int on) {
    if (!c) return QM_E_ARG;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    drop_events(c);
    c->timing = on != 0;
    return QM_OK;
}

extern "C" int qm_ctx_kernel_time(qm_ctx* c, const char* name, double* total_ms, int64_t* launches) {
    if (!c || !name) return QM_E_ARG;
    cudaSetDevice(c->device);
    double t = 0.0;
    int64_t n = 0;
    auto it = c->events.find(name);
    if (it != c->events.end()) {
        for (auto& pr : it->second) {
            QM_CHECK_CUDA(c, cudaEventSynchronize(pr.second));
            float ms = 0.f;
            QM_CHECK_CUDA(c, cudaEventElapsedTime(&ms, pr.first, pr.second));
            t += ms;
            n++;
        }
    }
    if (total_ms) *total_ms = t;
    if (launches) *launches = n;
    return QM_OK;
}

// ---------------------------------------------------------------------------
// RoPE table: src/convert.rs:161-176, same f32 formula
// ---------------------------------------------------------------------------
extern "C" int qm_rope_table(float theta, int rope_dim, int max_pos, float* cos_h, float* sin_h) {
    if (!cos_h || !sin_h || rope_dim <= 0 || (rope_dim & 1) || max_pos <= 0) return QM_E_ARG;
    int half = rope_dim / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; i++) {
        volatile float e = 2.0f * (float)i;     // keep the f32 rounding steps of the reference
        e = e / (float)rope_dim;
        freq[i] = 1.0f / powf(theta, e);
    }
    for (int pos = 0; pos < max_pos; pos++) {
        for (int i = 0; i < half; i++) {
            volatile float angle = (float)pos * freq[i];
            cos_h[(size_t)pos * half + i] = cosf(angle);
            sin_h[(size_t)pos * half + i] = sinf(angle);
        }
    }
    return QM_OK;
}

// ---------------------------------------------------------------------------
// DeltaNet state handles
// ---------------------------------------------------------------------------
static const size_t kConvPerSeq = (size_t)kConvSlots * kQKVDim;  // floats
static size_t s_per_seq(const qm_dn_state* st) { return (size_t)st->nvh * kHd * kHd; }  // floats

// V heads 2j and 2j+1 share QK head j, whose conv history the even head
// advances: a head range must start and end on a QK-head boundary.
static bool dn_heads_ok(int vh_lo, int nvh) {
    return vh_lo >= 0 && nvh >= 2 && vh_lo + nvh <= kNumV && (vh_lo % 2) == 0 && (nvh % 2) == 0;
}

extern "C" int qm_dn_state_create_heads(qm_ctx* c, int batch, int vh_lo, int nvh, qm_dn_state** out) {
    if (!c || !out || batch <= 0) return set_error(c, QM_E_ARG, "qm_dn_state_create: bad argument");
    if (!dn_heads_ok(vh_lo, nvh))
        return set_error(c, QM_E_ARG, "V-head range must be even-aligned within [0, 32)");
    *out = nullptr;
    cudaSetDevice(c->device);
    qm_dn_state* st = new (std::nothrow) qm_dn_state();
    if (!st) return QM_E_OOM;
    st->ctx = c;
    st->device = c->device;
    st->batch = batch;
    st->vh_lo = vh_lo;
    st->nvh = nvh;
    st->owned = true;
    if (cudaMalloc(&st->s, s_per_seq(st) * batch * 4) != cudaSuccess ||
        cudaMalloc(&st->conv, kConvPerSeq * batch * 4) != cudaSuccess) {
        if (st->s) cudaFree(st->s);
        delete st;
        return set_error(c, QM_E_OOM, "qm_dn_state_create: cudaMalloc failed");
    }
    int rc = qm_dn_state_reset(c, st);
    if (rc != QM_OK) {
        qm_dn_state_destroy(st);
        return rc;
    }
    *out = st;
    return QM_OK;
}

extern "C" int qm_dn_state_create(qm_ctx* c, int batch, qm_dn_state** out) {
    return qm_dn_state_create_heads(c, batch, 0, kNumV, out);
}

extern "C" int qm_dn_state_wrap_heads(qm_ctx* c, int batch, int vh_lo, int nvh, float* s, float* conv,
                                      qm_dn_state** out) {
    if (!c || !out || batch <= 0 || !s || !conv)
        return set_error(c, QM_E_ARG, "qm_dn_state_wrap: bad argument");
    if (!dn_heads_ok(vh_lo, nvh))
        return set_error(c, QM_E_ARG, "V-head range must be even-aligned within [0, 32)");
    if (((uintptr_t)s & 15) || ((uintptr_t)conv & 15))
        return set_error(c, QM_E_ARG, "qm_dn_state_wrap: storage must be 16-byte aligned");
    qm_dn_state* st = new (std::nothrow) qm_dn_state();
    if (!st) return QM_E_OOM;
    st->ctx = c;
    st->device = c->device;
    st->batch = batch;
    st->vh_lo = vh_lo;
    st->nvh = nvh;
    st->s = s;
    st->conv = conv;
    st->owned = false;
    *out = st;
    return QM_OK;
}

extern "C" int qm_dn_state_wrap(qm_ctx* c, int batch, float* s, float* conv, qm_dn_state** out) {
    return qm_dn_state_wrap_heads(c, batch, 0, kNumV, s, conv, out);
}

extern "C" int qm_dn_state_heads(const qm_dn_state* st, int* vh_lo, int* nvh) {
    if (!st) return QM_E_ARG;
    if (vh_lo) *vh_lo = st->vh_lo;
    if (nvh) *nvh = st->nvh;
    return QM_OK;
}

extern "C" int qm_dn_state_destroy(qm_dn_state* st) {
    if (!st) return QM_E_ARG;
    if (st->owned) {
        cudaSetDevice(st->device);  // cudaFree waits for work using the memory
        cudaFree(st->s);
        cudaFree(st->conv);
    }
    delete st;
    return QM_OK;
}

extern "C" int qm_dn_state_reset(qm_ctx* c, qm_dn_state* st) {
    if (!c || !st) return QM_E_ARG;
    if (st->ctx != c) return set_error(c, QM_E_MISMATCH, "state belongs to another context");
    cudaSetDevice(c->device);
    QM_CHECK_CUDA(c, cudaMemsetAsync(st->s, 0, s_per_seq(st) * st->batch * 4, c->stream));
    QM_CHECK_CUDA(c, cudaMemsetAsync(st->conv, 0, kConvPerSeq * st->batch * 4, c->stream));
    st->conv_pos = 0;
    return QM_OK;
}

extern "C" int qm_dn_state_snapshot(qm_ctx* c, const qm_dn_state* src, qm_dn_state** out) {
    if (!c || !src || !out) return QM_E_ARG;
    int rc = qm_dn_state_create_heads(c, src->batch, src->vh_lo, src->nvh, out);
    if (rc != QM_OK) return rc;
    rc = qm_dn_state_restore(c, *out, src);
    if (rc != QM_OK) {
        qm_dn_state_destroy(*out);
        *out = nullptr;
    }
    return rc;
}

extern "C" int qm_dn_state_restore(qm_ctx* c, qm_dn_state* dst, const qm_dn_state* src) {
    if (!c || !dst || !src) return QM_E_ARG;
    if (dst->batch != src->batch || dst->vh_lo != src->vh_lo || dst->nvh != src->nvh)
        return set_error(c, QM_E_MISMATCH, "restore: batch sizes or head ranges differ (reference: panic)");
    cudaSetDevice(c->device);
    QM_CHECK_CUDA(c, cudaMemcpyAsync(dst->s, src->s, s_per_seq(src) * src->batch * 4,
                                     cudaMemcpyDeviceToDevice, c->stream));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(dst->conv, src->conv, kConvPerSeq * src->batch * 4,
                                     cudaMemcpyDeviceToDevice, c->stream));
    dst->conv_pos = src->conv_pos;
    return QM_OK;
}

// Reference conv_buf[ch*3 + j] holds token conv_pos-3+j; the ring keeps
// token t in slot t % 4.
static inline int ring_slot(int64_t conv_pos, int j) {
    int64_t t = conv_pos - 3 + j;
    return (int)(((t % 4) + 4) % 4);
}

extern "C" int qm_dn_state_read(qm_ctx* c, const qm_dn_state* st, int b, float* s_h, float* conv_h) {
    if (!c || !st || b < 0 || b >= st->batch) return set_error(c, QM_E_ARG, "qm_dn_state_read: bad argument");
    cudaSetDevice(c->device);
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->stream));
    if (s_h)
        QM_CHECK_CUDA(c, cudaMemcpy(s_h, st->s + s_per_seq(st) * b, s_per_seq(st) * 4,
                                    cudaMemcpyDeviceToHost));
    if (conv_h) {
        std::vector<float> ring(kConvPerSeq);
        QM_CHECK_CUDA(c, cudaMemcpy(ring.data(), st->conv + kConvPerSeq * b, kConvPerSeq * 4,
                                    cudaMemcpyDeviceToHost));
        for (int j = 0; j < 3; j++) {
            const float* slot = ring.data() + (size_t)ring_slot(st->conv_pos, j) * kQKVDim;
            for (int ch = 0; ch < kQKVDim; ch++) conv_h[(size_t)ch * 3 + j] = slot[ch];
        }
    }
    return QM_OK;
}

extern "C" int qm_dn_state_write(qm_ctx* c, qm_dn_state* st, int b, const float* s_h,
                                 const float* conv_h) {
    if (!c || !st || b < 0 || b >= st->batch) return set_error(c, QM_E_ARG, "qm_dn_state_write: bad argument");
    cudaSetDevice(c->device);
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->stream));
    if (s_h)
        QM_CHECK_CUDA(c, cudaMemcpy(st->s + s_per_seq(st) * b, s_h, s_per_seq(st) * 4,
                                    cudaMemcpyHostToDevice));
    if (conv_h) {
        std::vector<float> ring(kConvPerSeq, 0.0f);
        for (int j = 0; j < 3; j++) {
            float* slot = ring.data() + (size_t)ring_slot(st->conv_pos, j) * kQKVDim;
            for (int ch = 0; ch < kQKVDim; ch++) slot[ch] = conv_h[(size_t)ch * 3 + j];
        }
        QM_CHECK_CUDA(c, cudaMemcpy(st->conv + kConvPerSeq * b, ring.data(), kConvPerSeq * 4,
                                    cudaMemcpyHostToDevice));
    }
    return QM_OK;
}

extern "C" int64_t qm_dn_state_conv_pos(const qm_dn_state* st) { return st ? st->conv_pos : -1; }
extern "C" int qm_dn_state_set_conv_pos(qm_dn_state* st, int64_t p) {
    if (!st || p < 0) return QM_E_ARG;
    st->conv_pos = p;
    return QM_OK;
}
extern "C" int qm_dn_state_batch(const qm_dn_state* st) { return st ? st->batch : -1; }
extern "C" int qm_dn_state_data(const qm_dn_state* st, float** s, float** conv) {
    if (!st) return QM_E_ARG;
    if (s) *s = st->s;
    if (conv) *conv = st->conv;
    return QM_OK;
}

// ---------------------------------------------------------------------------
// Pipelined host-buffer calls: the batch is cut into parts; part i's inputs
// are copied in on one stream, its kernels run on the context stream and its
// outputs are copied out on a third stream, so part i+1's input copy and part
// i-1's output copy overlap part i's kernels.  Measured on the 32-layer decode
// stack at batch 64: 2 parts 15.54 ms per step, 1 part 15.79, 4 parts 16.62
// (more parts cost more API calls and less efficient kernels than they hide).
// ---------------------------------------------------------------------------
static int ensure_pipe(qm_ctx* c) {
    if (c->pipe_ready) return QM_OK;
    QM_CHECK_CUDA(c, cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking));
    QM_CHECK_CUDA(c, cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking));
    for (int i = 0; i < 8; i++) {
        QM_CHECK_CUDA(c, cudaEventCreateWithFlags(&c->pipe_in[i], cudaEventDisableTiming));
        QM_CHECK_CUDA(c, cudaEventCreateWithFlags(&c->pipe_done[i], cudaEventDisableTiming));
    }
    QM_CHECK_CUDA(c, cudaHostAlloc(reinterpret_cast<void**>(&c->h_err), sizeof(int), cudaHostAllocDefault));
    c->pipe_ready = true;
    return QM_OK;
}

// kind 0: DeltaNet, 1: GQA.  Default: 2 parts from batch 8 up.
static int pipe_parts(const qm_ctx* c, int B, int kind) {
    int k = c->host_parts[kind] > 0 ? c->host_parts[kind] : (B >= 8 ? 2 : 1);
    return k < B ? k : B;
}

// Ends a pipelined call: the error word is copied behind the last output
// copy on the output stream (which already waits for the last kernel), so
// one synchronisation covers outputs and status.
static int pipe_finish(qm_ctx* c) {
    QM_CHECK_CUDA(c, cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->copy_out));
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->copy_out));
    const int err = *c->h_err;
    if (err) {
        cudaMemset(c->d_err, 0, sizeof(int));
        if (err & kErrBounds)
            return set_error(c, QM_E_RANGE, "a device-side index self-check failed (access skipped)");
        return set_error(c, QM_E_TIMEOUT, "a device-side bounded wait gave up (error word set)");
    }
    return QM_OK;
}

extern "C" int qm_ctx_set_host_parts(qm_ctx* c, int dn_parts, int gqa_parts) {
    if (!c) return QM_E_ARG;
    if (dn_parts < 0 || dn_parts > 8 || gqa_parts < 0 || gqa_parts > 8)
        return set_error(c, QM_E_ARG, "qm_ctx_set_host_parts: parts must be 0 (default) .. 8");
    c->host_parts[0] = dn_parts;
    c->host_parts[1] = gqa_parts;
    return QM_OK;
}

// Part i of k: sequences [b0, b0 + nb).
static void pipe_part(int B, int k, int i, int* b0, int* nb) {
    *b0 = (int)((int64_t)B * i / k);
    *nb = (int)((int64_t)B * (i + 1) / k) - *b0;
}

// ---------------------------------------------------------------------------
// DeltaNet decode
// ---------------------------------------------------------------------------
static int check_dn_params(qm_ctx* c, const qm_dn_params* p, bool need_gamma) {
    if (!p || !p->conv_w || !p->a_log || !p->dt_bias || (need_gamma && !p->norm_gamma))
        return set_error(c, QM_E_ARG, "DeltaNet params: null pointer");
    if ((uintptr_t)p->conv_w & 15) return set_error(c, QM_E_ARG, "conv_w must be 16-byte aligned");
    return QM_OK;
}

static int check_dn_decode(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st, const void* qkv,
                           const void* a, const void* b, const void* y, const void* z, const void* out) {
    if (!c) return QM_E_ARG;
    if (!st || !qkv || !a || !b || (!y && !out) || (out && !z) || (z && !out))
        return set_error(c, QM_E_ARG, "qm_dn_decode: null pointer (y or z+out required)");
    if (st->ctx != c) return set_error(c, QM_E_MISMATCH, "state belongs to another context");
    return check_dn_params(c, p, z != nullptr);
}

extern "C" int qm_dn_decode(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                            const float* a, const float* b, float* y, const float* z, float* out) {
    int rc = check_dn_decode(c, p, st, qkv, a, b, y, z, out);
    if (rc) return rc;
    if (((uintptr_t)qkv & 15)) return set_error(c, QM_E_ARG, "qkv must be 16-byte aligned");
    cudaSetDevice(c->device);
    cudaError_t e = launch_dn_decode(c, p, st, qkv, a, b, y, z, out);
    if (e != cudaSuccess) return cuda_error(c, e, "dn_decode launch");
    st->conv_pos += 1;
    return QM_OK;
}

// T sequential decode steps in one launch, the state kept on chip (dn_decode_seq.cu).
extern "C" int qm_dn_decode_seq(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st, int T,
                                const float* qkv, const float* a, const float* b, float* y,
                                const float* z, float* out) {
    int rc = check_dn_decode(c, p, st, qkv, a, b, y, z, out);
    if (rc) return rc;
    if (T <= 0) return set_error(c, QM_E_ARG, "qm_dn_decode_seq: T <= 0");
    if (((uintptr_t)qkv & 15) || (z && ((uintptr_t)z & 15)))
        return set_error(c, QM_E_ARG, "qm_dn_decode_seq: qkv and z must be 16-byte aligned");
    cudaSetDevice(c->device);
    cudaError_t e = launch_dn_decode_seq(c, p, st, T, qkv, a, b, y, z, out);
    if (e != cudaSuccess) return cuda_error(c, e, "dn_decode_seq launch");
    st->conv_pos += T;
    return QM_OK;
}

extern "C" int qm_dn_decode_host(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st,
                                 const float* qkv, const float* a, const float* b, float* y,
                                 const float* z, float* out) {
    int rc = check_dn_decode(c, p, st, qkv, a, b, y, z, out);
    if (rc) return rc;
    const size_t B = st->batch;
    // inputs are full width; y and out cover the state's V heads
    const size_t n_qkv = B * kQKVDim, n_ab = B * kNumV, n_z = B * kVDim, n_y = B * st->nvh * kHd;
    size_t bytes = 4 * (n_qkv + 2 * n_ab + (y ? n_y : 0) + (z ? n_z + n_y : 0)) + 256 * 6;
    cudaSetDevice(c->device);
    rc = ensure_stage(c, bytes);
    if (!rc) rc = ensure_pipe(c);
    if (rc) return rc;
    char* base = (char*)c->stage;
    auto carve = [&](size_t n) {
        float* r = (float*)base;
        base += (n * 4 + 255) & ~size_t(255);
        return r;
    };
    if (c->host_direct) {
        // every buffer page-locked and mapped: one launch reads the inputs and
        // writes the outputs in place over PCIe (measured at batch 64: 130 us
        // per call against 168 us staged in two overlapped parts, and 153-170 us
        // with qkv still brought in by copy engine and the rest in place)
        const void* m_qkv = mapped_host(qkv, n_qkv * 4);
        const void* m_a = mapped_host(a, n_ab * 4);
        const void* m_b = mapped_host(b, n_ab * 4);
        const void* m_z = z ? mapped_host(z, n_z * 4) : nullptr;
        void* m_y = y ? mapped_host(y, n_y * 4) : nullptr;
        void* m_out = out ? mapped_host(out, n_y * 4) : nullptr;
        if (m_qkv && m_a && m_b && (!z || m_z) && (!y || m_y) && (!out || m_out) &&
            ((uintptr_t)m_qkv & 15) == 0) {
            cudaError_t e = launch_dn_decode(c, p, st, (const float*)m_qkv, (const float*)m_a,
                                             (const float*)m_b, (float*)m_y, (const float*)m_z,
                                             (float*)m_out, 0, -1, true);
            if (e != cudaSuccess) return cuda_error(c, e, "dn_decode launch");
            st->conv_pos += 1;
            c->host_in_place += 1;
            return direct_finish(c);
        }
    }
    c->host_staged += 1;
    float* d_qkv = carve(n_qkv);
    float* d_a = carve(n_ab);
    float* d_b = carve(n_ab);
    float* d_y = y ? carve(n_y) : nullptr;
    float* d_z = z ? carve(n_z) : nullptr;
    float* d_out = z ? carve(n_y) : nullptr;
    const size_t ny = (size_t)st->nvh * kHd;  // y / out floats per sequence
    const int k = pipe_parts(c, (int)B, 0);
    // the input copies must not overtake work already queued on the context stream
    QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_done[7], c->stream));
    QM_CHECK_CUDA(c, cudaStreamWaitEvent(c->copy_in, c->pipe_done[7], 0));
    for (int i = 0; i < k; i++) {
        int b0, nb;
        pipe_part((int)B, k, i, &b0, &nb);
        cudaStream_t in = c->copy_in, out_s = c->copy_out;
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_qkv + (size_t)b0 * kQKVDim, qkv + (size_t)b0 * kQKVDim,
                                         (size_t)nb * kQKVDim * 4, cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_a + (size_t)b0 * kNumV, a + (size_t)b0 * kNumV,
                                         (size_t)nb * kNumV * 4, cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_b + (size_t)b0 * kNumV, b + (size_t)b0 * kNumV,
                                         (size_t)nb * kNumV * 4, cudaMemcpyHostToDevice, in));
        if (z)
            QM_CHECK_CUDA(c, cudaMemcpyAsync(d_z + (size_t)b0 * kVDim, z + (size_t)b0 * kVDim,
                                             (size_t)nb * kVDim * 4, cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_in[i], in));
        QM_CHECK_CUDA(c, cudaStreamWaitEvent(c->stream, c->pipe_in[i], 0));
        cudaError_t e = launch_dn_decode(c, p, st, d_qkv, d_a, d_b, d_y, d_z, d_out, b0, nb);
        if (e != cudaSuccess) return cuda_error(c, e, "dn_decode launch");
        QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_done[i], c->stream));
        QM_CHECK_CUDA(c, cudaStreamWaitEvent(out_s, c->pipe_done[i], 0));
        if (y)
            QM_CHECK_CUDA(c, cudaMemcpyAsync(y + b0 * ny, d_y + b0 * ny, nb * ny * 4, cudaMemcpyDeviceToHost,
                                             out_s));
        if (out)
            QM_CHECK_CUDA(c, cudaMemcpyAsync(out + b0 * ny, d_out + b0 * ny, nb * ny * 4,
                                             cudaMemcpyDeviceToHost, out_s));
    }
    st->conv_pos += 1;
    return pipe_finish(c);
}

// ---------------------------------------------------------------------------
// KV cache handles
// ---------------------------------------------------------------------------
static size_t kv_elems(int batch, int nkv, int cap) { return (size_t)batch * nkv * cap * kD; }

extern "C" int qm_kv_create_heads(qm_ctx* c, int batch, int capacity, int kv_lo, int nkv, qm_kv** out) {
    if (!c || !out || batch <= 0 || capacity <= 0)
        return set_error(c, QM_E_ARG, "qm_kv_create: bad argument");
    if (kv_lo < 0 || nkv < 1 || kv_lo + nkv > kNumKVH)
        return set_error(c, QM_E_ARG, "KV-head range outside [0, 4)");
    *out = nullptr;
    cudaSetDevice(c->device);
    qm_kv* kv = new (std::nothrow) qm_kv();
    if (!kv) return QM_E_OOM;
    kv->ctx = c;
    kv->device = c->device;
    kv->batch = batch;
    kv->capacity = capacity;
    kv->kv_lo = kv_lo;
    kv->nkv = nkv;
    kv->owned = true;
    size_t bytes = kv_elems(batch, nkv, capacity) * 2;
    if (cudaMalloc(&kv->k, bytes) != cudaSuccess || cudaMalloc(&kv->v, bytes) != cudaSuccess) {
        if (kv->k) cudaFree(kv->k);
        delete kv;
        return set_error(c, QM_E_OOM, "qm_kv_create: cudaMalloc failed");
    }
    cudaMemsetAsync(kv->k, 0, bytes, c->stream);
    cudaMemsetAsync(kv->v, 0, bytes, c->stream);
    int rc = make_kv_tmaps(kv);
    if (rc) {
        qm_kv_destroy(kv);
        return rc;
    }
    *out = kv;
    return QM_OK;
}

extern "C" int qm_kv_create(qm_ctx* c, int batch, int capacity, qm_kv** out) {
    return qm_kv_create_heads(c, batch, capacity, 0, kNumKVH, out);
}

extern "C" int qm_kv_wrap_heads(qm_ctx* c, int batch, int capacity, int kv_lo, int nkv, uint16_t* k,
                                uint16_t* v, qm_kv** out) {
    if (!c || !out || batch <= 0 || capacity <= 0 || !k || !v)
        return set_error(c, QM_E_ARG, "qm_kv_wrap: bad argument");
    if (kv_lo < 0 || nkv < 1 || kv_lo + nkv > kNumKVH)
        return set_error(c, QM_E_ARG, "KV-head range outside [0, 4)");
    if (((uintptr_t)k & 15) || ((uintptr_t)v & 15))
        return set_error(c, QM_E_ARG, "qm_kv_wrap: cache must be 16-byte aligned");
    qm_kv* kv = new (std::nothrow) qm_kv();
    if (!kv) return QM_E_OOM;
    kv->ctx = c;
    kv->device = c->device;
    kv->batch = batch;
    kv->capacity = capacity;
    kv->kv_lo = kv_lo;
    kv->nkv = nkv;
    kv->k = k;
    kv->v = v;
    kv->owned = false;
    int rc = make_kv_tmaps(kv);
    if (rc) {
        delete kv;
        return rc;
    }
    *out = kv;
    return QM_OK;
}

extern "C" int qm_kv_wrap(qm_ctx* c, int batch, int capacity, uint16_t* k, uint16_t* v, qm_kv** out) {
    return qm_kv_wrap_heads(c, batch, capacity, 0, kNumKVH, k, v, out);
}

extern "C" int qm_kv_heads(const qm_kv* kv, int* kv_lo, int* nkv) {
    if (!kv) return QM_E_ARG;
    if (kv_lo) *kv_lo = kv->kv_lo;
    if (nkv) *nkv = kv->nkv;
    return QM_OK;
}

extern "C" int qm_kv_destroy(qm_kv* kv) {
    if (!kv) return QM_E_ARG;
    if (kv->owned) {
        cudaSetDevice(kv->device);  // cudaFree waits for work using the memory
        cudaFree(kv->k);
        cudaFree(kv->v);
    }
    delete kv;
    return QM_OK;
}

extern "C" int qm_kv_snapshot(qm_ctx* c, const qm_kv* src, qm_kv** out) {
    if (!c || !src || !out) return QM_E_ARG;
    int rc = qm_kv_create_heads(c, src->batch, src->capacity, src->kv_lo, src->nkv, out);
    if (rc) return rc;
    rc = qm_kv_restore(c, *out, src);
    if (rc) {
        qm_kv_destroy(*out);
        *out = nullptr;
    }
    return rc;
}

extern "C" int qm_kv_restore(qm_ctx* c, qm_kv* dst, const qm_kv* src) {
    if (!c || !dst || !src) return QM_E_ARG;
    if (dst->batch != src->batch || dst->capacity < src->seq_len || dst->kv_lo != src->kv_lo ||
        dst->nkv != src->nkv)
        return set_error(c, QM_E_MISMATCH, "kv restore: batch, capacity or head-range mismatch");
    cudaSetDevice(c->device);
    // Copy the filled prefix of every (sequence, kv-head) row block.
    size_t row = (size_t)kD * 2;
    QM_CHECK_CUDA(c, cudaMemcpy2DAsync(dst->k, (size_t)dst->capacity * row, src->k,
                                       (size_t)src->capacity * row, (size_t)src->seq_len * row,
                                       (size_t)src->batch * src->nkv, cudaMemcpyDeviceToDevice,
                                       c->stream));
    QM_CHECK_CUDA(c, cudaMemcpy2DAsync(dst->v, (size_t)dst->capacity * row, src->v,
                                       (size_t)src->capacity * row, (size_t)src->seq_len * row,
                                       (size_t)src->batch * src->nkv, cudaMemcpyDeviceToDevice,
                                       c->stream));
    dst->seq_len = src->seq_len;
    return QM_OK;
}

extern "C" int64_t qm_kv_seq_len(const qm_kv* kv) { return kv ? kv->seq_len : -1; }
extern "C" int qm_kv_set_seq_len(qm_kv* kv, int64_t n) {
    if (!kv || n < 0 || n > kv->capacity) return QM_E_ARG;
    kv->seq_len = n;
    return QM_OK;
}
extern "C" int qm_kv_capacity(const qm_kv* kv) { return kv ? kv->capacity : -1; }
extern "C" int qm_kv_batch(const qm_kv* kv) { return kv ? kv->batch : -1; }
extern "C" int qm_kv_data(const qm_kv* kv, uint16_t** k, uint16_t** v) {
    if (!kv) return QM_E_ARG;
    if (k) *k = kv->k;
    if (v) *v = kv->v;
    return QM_OK;
}

// ---------------------------------------------------------------------------
// GQA decode
// ---------------------------------------------------------------------------
static int check_gqa_params(qm_ctx* c, const qm_gqa_params* p) {
    if (!p || !p->q_norm || !p->k_norm || !p->rope_cos || !p->rope_sin || p->max_pos <= 0)
        return set_error(c, QM_E_ARG, "GQA params: null pointer or max_pos <= 0");
    return QM_OK;
}

extern "C" int qm_gqa_decode(qm_ctx* c, const qm_gqa_params* p, qm_kv* kv, const float* q_gate,
                             const float* k_new, const float* v_new, float* out) {
    if (!c) return QM_E_ARG;
    if (!kv || !q_gate || !k_new || !v_new || !out)
        return set_error(c, QM_E_ARG, "qm_gqa_decode: null pointer");
    if (kv->ctx != c) return set_error(c, QM_E_MISMATCH, "cache belongs to another context");
    int rc = check_gqa_params(c, p);
    if (rc) return rc;
    if (kv->seq_len >= kv->capacity)
        return set_error(c, QM_E_RANGE, "qm_gqa_decode: KV cache full");
    if (kv->seq_len >= p->max_pos)
        return set_error(c, QM_E_RANGE, "qm_gqa_decode: position beyond the RoPE table");
    cudaSetDevice(c->device);
    size_t ws = gqa_decode_ws_bytes(kv->batch, kv->nkv, kv->seq_len, c->num_sms);
    rc = ensure_workspace(c, ws);
    if (rc) return rc;
    cudaError_t e = launch_gqa_decode(c, p, kv, q_gate, k_new, v_new, out, c->ws, c->ws_bytes);
    if (e != cudaSuccess) return cuda_error(c, e, "gqa_decode launch");
    kv->seq_len += 1;
    return QM_OK;
}

extern "C" int qm_gqa_decode_host(qm_ctx* c, const qm_gqa_params* p, qm_kv* kv,
                                  const float* q_gate, const float* k_new, const float* v_new,
                                  float* out) {
    if (!c) return QM_E_ARG;
    if (!kv || !q_gate || !k_new || !v_new || !out)
        return set_error(c, QM_E_ARG, "qm_gqa_decode_host: null pointer");
    if (kv->ctx != c) return set_error(c, QM_E_MISMATCH, "cache belongs to another context");
    int rc = check_gqa_params(c, p);
    if (rc) return rc;
    if (kv->seq_len >= kv->capacity) return set_error(c, QM_E_RANGE, "qm_gqa_decode: KV cache full");
    if (kv->seq_len >= p->max_pos)
        return set_error(c, QM_E_RANGE, "qm_gqa_decode: position beyond the RoPE table");
    const int B = kv->batch;
    const size_t qrow = (size_t)kNumH * 2 * kD, kvrow = (size_t)kNumKVH * kD,
                 orow = (size_t)kv->nkv * kGroup * kD;  // out covers the cache's heads
    const size_t n_q = B * qrow, n_kv = B * kvrow, n_o = B * orow;
    cudaSetDevice(c->device);
    rc = ensure_stage(c, 4 * (n_q + 2 * n_kv + n_o) + 1024);
    if (!rc) rc = ensure_pipe(c);
    if (rc) return rc;
    if (c->host_direct) {
        const void* m_q = mapped_host(q_gate, n_q * 4);
        const void* m_k = mapped_host(k_new, n_kv * 4);
        const void* m_v = mapped_host(v_new, n_kv * 4);
        void* m_o = mapped_host(out, n_o * 4);
        if (m_q && m_k && m_v && m_o) {
            c->host_in_place += 1;
            rc = ensure_workspace(c, gqa_decode_ws_bytes(B, kv->nkv, kv->seq_len, c->num_sms));
            if (rc) return rc;
            // prep reads q, k_new, v_new in place; the gate halves of q_gate and
            // v_new, which combine needs after the attention, come into device
            // memory by copy engine while the attention runs (same layout, so
            // combine indexes them as it would the inputs)
            float* d_q = (float*)c->stage;
            float* d_v = (float*)((char*)c->stage + ((n_q * 4 + 255) & ~size_t(255)));
            QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_done[7], c->stream));
            QM_CHECK_CUDA(c, cudaStreamWaitEvent(c->copy_in, c->pipe_done[7], 0));
            QM_CHECK_CUDA(c, cudaMemcpy2DAsync(d_q + kD, 2 * kD * 4, q_gate + kD, 2 * kD * 4, kD * 4,
                                               (size_t)B * kNumH, cudaMemcpyHostToDevice, c->copy_in));
            QM_CHECK_CUDA(c, cudaMemcpyAsync(d_v, v_new, n_kv * 4, cudaMemcpyHostToDevice, c->copy_in));
            QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_in[0], c->copy_in));
            GqaCombineSrc comb;
            comb.q_gate = d_q;
            comb.v_new = d_v;
            comb.ready = c->pipe_in[0];
            cudaError_t e = launch_gqa_decode(c, p, kv, (const float*)m_q, (const float*)m_k,
                                              (const float*)m_v, (float*)m_o, c->ws, c->ws_bytes, 0, -1,
                                              &comb);
            if (e != cudaSuccess) return cuda_error(c, e, "gqa_decode launch");
            kv->seq_len += 1;
            return direct_finish(c);
        }
    }
    c->host_staged += 1;
    const int k = pipe_parts(c, B, 1);
    int smallest = B;  // the smallest part needs the most split-KV partials
    for (int i = 0; i < k; i++) {
        int b0, nb;
        pipe_part(B, k, i, &b0, &nb);
        smallest = nb < smallest ? nb : smallest;
    }
    rc = ensure_workspace(c, gqa_decode_ws_bytes(B, kv->nkv, kv->seq_len, c->num_sms, smallest));
    if (rc) return rc;
    char* base = (char*)c->stage;
    auto carve = [&](size_t n) {
        float* r = (float*)base;
        base += (n * 4 + 255) & ~size_t(255);
        return r;
    };
    float* d_q = carve(n_q);
    float* d_k = carve(n_kv);
    float* d_v = carve(n_kv);
    float* d_o = carve(n_o);
    QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_done[7], c->stream));
    QM_CHECK_CUDA(c, cudaStreamWaitEvent(c->copy_in, c->pipe_done[7], 0));
    for (int i = 0; i < k; i++) {
        int b0, nb;
        pipe_part(B, k, i, &b0, &nb);
        cudaStream_t in = c->copy_in, out_s = c->copy_out;
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_q + b0 * qrow, q_gate + b0 * qrow, nb * qrow * 4,
                                         cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_k + b0 * kvrow, k_new + b0 * kvrow, nb * kvrow * 4,
                                         cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaMemcpyAsync(d_v + b0 * kvrow, v_new + b0 * kvrow, nb * kvrow * 4,
                                         cudaMemcpyHostToDevice, in));
        QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_in[i], in));
        QM_CHECK_CUDA(c, cudaStreamWaitEvent(c->stream, c->pipe_in[i], 0));
        cudaError_t e = launch_gqa_decode(c, p, kv, d_q, d_k, d_v, d_o, c->ws, c->ws_bytes, b0, nb);
        if (e != cudaSuccess) return cuda_error(c, e, "gqa_decode launch");
        QM_CHECK_CUDA(c, cudaEventRecord(c->pipe_done[i], c->stream));
        QM_CHECK_CUDA(c, cudaStreamWaitEvent(out_s, c->pipe_done[i], 0));
        QM_CHECK_CUDA(c, cudaMemcpyAsync(out + b0 * orow, d_o + b0 * orow, nb * orow * 4,
                                         cudaMemcpyDeviceToHost, out_s));
    }
    kv->seq_len += 1;
    return pipe_finish(c);
}


// ---------------------------------------------------------------------------
// Prefill on host buffers.  The reference's GPU prefill moves every layer's
// activations between host and device around its recurrence
// (src/gpu_inference.rs:464-476 down, 591-604 up); these calls take the host
// buffers, copy them in on the context stream, run the device prefill and
// copy the outputs back before returning.  Prefill kernels read their
// inputs many times, so the inputs are always staged (never read over PCIe
// in place).
// ---------------------------------------------------------------------------
static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" int qm_dn_prefill_host(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st, int T,
                                  const uint16_t* qkv, const float* a, const float* b, float* y,
                                  const float* z, float* out) {
    if (!c) return QM_E_ARG;
    if (!st || !qkv || !a || !b || !y || T <= 0 || (out && !z) || (z && !out))
        return set_error(c, QM_E_ARG, "qm_dn_prefill_host: null pointer, T <= 0, or out without z");
    if (st->ctx != c) return set_error(c, QM_E_MISMATCH, "state belongs to another context");
    const size_t n = (size_t)st->batch * (size_t)T;
    const size_t b_qkv = n * kQKVDim * 2, b_ab = n * kNumV * 4, b_y = n * kVDim * 4;
    const size_t bytes = al256(b_qkv) + 2 * al256(b_ab) + al256(b_y) + (z ? 2 * al256(b_y) : 0);
    cudaSetDevice(c->device);
    int rc = ensure_stage(c, bytes);
    if (!rc) rc = ensure_pipe(c);
    if (rc) return rc;
    char* base = static_cast<char*>(c->stage);
    auto carve = [&](size_t nb) {
        char* r = base;
        base += al256(nb);
        return r;
    };
    uint16_t* d_qkv = reinterpret_cast<uint16_t*>(carve(b_qkv));
    float* d_a = reinterpret_cast<float*>(carve(b_ab));
    float* d_b = reinterpret_cast<float*>(carve(b_ab));
    float* d_y = reinterpret_cast<float*>(carve(b_y));
    float* d_z = z ? reinterpret_cast<float*>(carve(b_y)) : nullptr;
    float* d_out = z ? reinterpret_cast<float*>(carve(b_y)) : nullptr;
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_qkv, qkv, b_qkv, cudaMemcpyHostToDevice, c->stream));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_a, a, b_ab, cudaMemcpyHostToDevice, c->stream));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_b, b, b_ab, cudaMemcpyHostToDevice, c->stream));
    if (z) QM_CHECK_CUDA(c, cudaMemcpyAsync(d_z, z, b_y, cudaMemcpyHostToDevice, c->stream));
    rc = qm_dn_prefill(c, p, st, T, d_qkv, d_a, d_b, d_y, d_z, d_out);
    if (rc) return rc;
    QM_CHECK_CUDA(c, cudaMemcpyAsync(y, d_y, b_y, cudaMemcpyDeviceToHost, c->stream));
    if (out) QM_CHECK_CUDA(c, cudaMemcpyAsync(out, d_out, b_y, cudaMemcpyDeviceToHost, c->stream));
    c->host_staged += 1;
    return direct_finish(c);
}

extern "C" int qm_gqa_prefill_host(qm_ctx* c, const qm_gqa_params* p, qm_kv* kv, int T,
                                   const uint16_t* q_gate, const uint16_t* k, const uint16_t* v,
                                   float* out) {
    if (!c) return QM_E_ARG;
    if (!kv || !q_gate || !k || !v || !out || T <= 0)
        return set_error(c, QM_E_ARG, "qm_gqa_prefill_host: null pointer or T <= 0");
    if (kv->ctx != c) return set_error(c, QM_E_MISMATCH, "cache belongs to another context");
    const size_t n = (size_t)kv->batch * (size_t)T;
    const size_t b_q = n * kNumH * 2 * kD * 2, b_kv = n * kNumKVH * kD * 2, b_o = n * kNumH * kD * 4;
    const size_t bytes = al256(b_q) + 2 * al256(b_kv) + al256(b_o);
    cudaSetDevice(c->device);
    int rc = ensure_stage(c, bytes);
    if (!rc) rc = ensure_pipe(c);
    if (rc) return rc;
    char* base = static_cast<char*>(c->stage);
    uint16_t* d_q = reinterpret_cast<uint16_t*>(base);
    uint16_t* d_k = reinterpret_cast<uint16_t*>(base + al256(b_q));
    uint16_t* d_v = reinterpret_cast<uint16_t*>(base + al256(b_q) + al256(b_kv));
    float* d_o = reinterpret_cast<float*>(base + al256(b_q) + 2 * al256(b_kv));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_q, q_gate, b_q, cudaMemcpyHostToDevice, c->stream));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_k, k, b_kv, cudaMemcpyHostToDevice, c->stream));
    QM_CHECK_CUDA(c, cudaMemcpyAsync(d_v, v, b_kv, cudaMemcpyHostToDevice, c->stream));
    rc = qm_gqa_prefill(c, p, kv, T, d_q, d_k, d_v, d_o);
    if (rc) return rc;
    QM_CHECK_CUDA(c, cudaMemcpyAsync(out, d_o, b_o, cudaMemcpyDeviceToHost, c->stream));
    c->host_staged += 1;
    return direct_finish(c);
}
