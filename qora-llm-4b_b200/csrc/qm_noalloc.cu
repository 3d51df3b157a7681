// qm_gqa_decode_noalloc: GQA decode with no device allocation at all.
//
// Some callers of this library cannot call cudaMalloc: an inference server
// whose memory manager reserves all of HBM at start-up and forbids
// allocations afterwards (a late cudaMalloc may fail under memory pressure
// and synchronises the device), or a plugin that only borrows the host
// engine's buffers and stream and owns no device memory.  They cannot create
// a qm_ctx (which allocates an error word and a workspace) nor let
// qm_gqa_decode grow the workspace.  This entry point serves them: the
// caller passes the KV cache, the inputs, the output and a stream; the
// split-KV partials live in a fixed array in this file.
//
// The array is `static __device__`, so every GPU that loads the library
// holds QM_NOALLOC_SCRATCH_BYTES of it until the process exits.  Host code
// cannot use its name as a device address; the first call on each device
// looks the address up with cudaGetSymbolAddress and keeps it.
#include <mutex>

#include "qm_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[QM_NOALLOC_SCRATCH_BYTES];

// The last 256 bytes hold the device-side error word; the rest is workspace.
constexpr size_t kErrBytes = 256;
constexpr size_t kWsBytes = QM_NOALLOC_SCRATCH_BYTES - kErrBytes;

struct DeviceSetup {
    bool done = false;
    void* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

// Runs once per device, with that device current.
int setup_device(int dev, DeviceSetup** out) {
    if (dev < 0 || dev >= kMaxDevices) return QM_E_ARG;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.done) {
        int major = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return QM_E_CUDA;
        if (major != 10) return QM_E_UNSUPPORTED;
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
            return QM_E_CUDA;
        s.scratch = p;
        s.num_sms = sms;
        s.done = true;
    }
    *out = &s;
    return QM_OK;
}

}  // namespace

extern "C" int qm_gqa_decode_noalloc(const qm_gqa_params* p, uint16_t* k_cache, uint16_t* v_cache,
                                     int batch, int capacity, int64_t seq_len,
                                     const float* q_gate, const float* k_new, const float* v_new,
                                     float* out, void* stream) {
    if (!p || !p->q_norm || !p->k_norm || !p->rope_cos || !p->rope_sin || p->max_pos <= 0 ||
        !k_cache || !v_cache || !q_gate || !k_new || !v_new || !out || batch <= 0 ||
        capacity <= 0 || seq_len < 0)
        return QM_E_ARG;
    if (((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15)) return QM_E_ARG;
    if (seq_len >= capacity || seq_len >= p->max_pos) return QM_E_RANGE;

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QM_E_CUDA;
    DeviceSetup* s = nullptr;
    int rc = setup_device(dev, &s);
    if (rc != QM_OK) return rc;
    // Reject what does not fit the fixed scratch (never grow it).
    if (qm::gqa_decode_ws_bytes(batch, qm::kNumKVH, seq_len, s->num_sms) > kWsBytes) return QM_E_SHAPE;

    // Host-side bookkeeping only: these objects own no device memory.
    qm_ctx c;
    c.device = dev;
    c.stream = static_cast<cudaStream_t>(stream);
    c.num_sms = s->num_sms;
    c.d_err = reinterpret_cast<int*>(static_cast<char*>(s->scratch) + kWsBytes);
    qm_kv kv;
    kv.ctx = &c;
    kv.device = dev;
    kv.batch = batch;
    kv.capacity = capacity;
    kv.k = k_cache;
    kv.v = v_cache;
    kv.seq_len = seq_len;
    if (qm::make_kv_tmaps(&kv) != QM_OK) return QM_E_CUDA;

    // The error word must start at zero; the partials are fully rewritten.
    if (cudaMemsetAsync(c.d_err, 0, sizeof(int), c.stream) != cudaSuccess) return QM_E_CUDA;
    cudaError_t e =
        qm::launch_gqa_decode(&c, p, &kv, q_gate, k_new, v_new, out, s->scratch, kWsBytes);
    return e == cudaSuccess ? QM_OK : QM_E_CUDA;
}
