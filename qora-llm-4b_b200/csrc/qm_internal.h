// Internal definitions shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "qora_mixer.h"

namespace qm {

// Qor4bConfig::default_4b mixer fields (src/config.rs:52-78).
constexpr int kNumQK = 16;
constexpr int kNumV = 32;
constexpr int kHd = 128;                            // DeltaNet head dim
constexpr int kConvK = 4;
constexpr int kQDim = kNumQK * kHd;                 // 2048
constexpr int kVDim = kNumV * kHd;                  // 4096
constexpr int kQKVDim = 2 * kQDim + kVDim;          // 8192
constexpr int kConvSlots = 4;                       // ring of the last 4 inputs
constexpr int kNumH = 16;                           // attention Q heads
constexpr int kNumKVH = 4;
constexpr int kD = 256;                             // attention head dim
constexpr int kGroup = kNumH / kNumKVH;             // 4
constexpr int kRot = 64;                            // rope_dim
constexpr int kHalfRot = kRot / 2;                  // 32

// Device-side error word bits: a bounded wait gave up; an index self-check failed.
constexpr int kErrTimeout = 1;
constexpr int kErrBounds = 2;

}  // namespace qm

struct qm_ctx {
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int* d_err = nullptr;           // device error word
    void* ws = nullptr;             // workspace (split-KV partials, staging)
    size_t ws_bytes = 0;
    int num_sms = 0;
    int64_t launches = 0;
    std::string last_error;
    // host-staging for the _host variants (device side)
    void* stage = nullptr;
    size_t stage_bytes = 0;
    // optional per-kernel CUDA-event timing (qm_ctx_set_timing)
    bool timing = false;
    std::map<std::string, std::vector<std::pair<cudaEvent_t, cudaEvent_t>>> events;
    std::vector<cudaEvent_t> event_pool;
    // copy streams and events of the pipelined _host variants (created on first use)
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    cudaEvent_t pipe_in[8] = {}, pipe_done[8] = {};
    bool pipe_ready = false;
    int* h_err = nullptr;           // pinned copy of the error word (pipelined calls)
    int host_parts[2] = {0, 0};     // parts of a DeltaNet / GQA _host call (0: default)
    bool host_direct = true;        // _host calls use page-locked buffers in place
    int64_t host_in_place = 0, host_staged = 0;  // _host calls by path
    // qm_gemv: per-CTA partial sums of a column tile and the per-tile counters
    void* gemv_partial = nullptr;
    size_t gemv_partial_bytes = 0;
    int* gemv_count = nullptr;
};

struct qm_dn_state {
    qm_ctx* ctx = nullptr;
    int device = 0;           // destroy uses this, never ctx (ctx may be gone)
    int batch = 0;
    int vh_lo = 0;            // V heads [vh_lo, vh_lo + nvh) of the model (head shard)
    int nvh = qm::kNumV;
    float* s = nullptr;       // [B, nvh, 128, 128]
    float* conv = nullptr;    // [B, 4, 8192] ring, token t in slot t % 4
    int64_t conv_pos = 0;
    bool owned = false;
};

struct qm_kv {
    qm_ctx* ctx = nullptr;
    int device = 0;           // destroy uses this, never ctx (ctx may be gone)
    int batch = 0;
    int capacity = 0;
    int kv_lo = 0;            // KV heads [kv_lo, kv_lo + nkv) of the model (head shard)
    int nkv = qm::kNumKVH;
    uint16_t* k = nullptr;    // [B, nkv, cap, 256] bf16
    uint16_t* v = nullptr;
    int64_t seq_len = 0;
    bool owned = false;
    CUtensorMap tmap_k;       // 3-D view {256, cap, B*nkv}, box {64, 64, 1}, 128B swizzle
    CUtensorMap tmap_v;
    bool tmaps_ok = false;
};

namespace qm {

int set_error(qm_ctx* ctx, int code, const std::string& msg);
// y[b][v] = x[b] . W[v] for QM_W_F16_ROWS / QM_W_Q4_ROWS weights (qm_head.cu)
int gemv_rows(qm_ctx* c, const qm_weight* w, int batch, const float* x, float* y);
// the split-K scratch the GEMV and the GEMM share (calls on one context are stream-ordered): at least
// partial_bytes of f32 partials and kSplitCounters zeroed tile counters, which every launch leaves zeroed
constexpr int kSplitCounters = 4096;
int ensure_gemv_scratch(qm_ctx* c, size_t partial_bytes);
int cuda_error(qm_ctx* ctx, cudaError_t e, const char* what);
int ensure_workspace(qm_ctx* ctx, size_t bytes);
int ensure_stage(qm_ctx* ctx, size_t bytes);
int make_kv_tmaps(qm_kv* kv);

// Records a start/stop event pair around a launch when ctx->timing is on.
struct TimedLaunch {
    qm_ctx* ctx;
    cudaEvent_t stop = nullptr;
    TimedLaunch(qm_ctx* c, const char* name);
    ~TimedLaunch();
};

// Kernel launchers (return cudaError_t from the launch).
// b0, nb: run sequences [b0, b0 + nb) of the handle's batch (nb < 0: all)
// pair: fetch q and k once per V-head pair (inputs in host memory, read over PCIe)
cudaError_t launch_dn_decode(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                             const float* a, const float* b, float* y, const float* z, float* out,
                             int b0 = 0, int nb = -1, bool pair = false);
// T tokens per sequence in order, the state in registers for the whole call
cudaError_t launch_dn_decode_seq(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                                 const float* qkv, const float* a, const float* b, float* y,
                                 const float* z, float* out);
// GqaCombineSrc: where the combine kernel reads the gate half of q_gate and
// v_new (default: the call's own q_gate / v_new), after waiting for `ready`
// on the launch stream when it is set.
struct GqaCombineSrc {
    const float* q_gate = nullptr;
    const float* v_new = nullptr;
    cudaEvent_t ready = nullptr;
};
cudaError_t launch_gqa_decode(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, const float* q_gate,
                              const float* k_new, const float* v_new, float* out, void* ws,
                              size_t ws_bytes, int b0 = 0, int nb = -1,
                              const GqaCombineSrc* comb = nullptr);
size_t gqa_decode_ws_bytes(int batch, int nkv, int64_t seq_len, int num_sms, int nb = -1);
cudaError_t launch_gqa_prefill(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, int T,
                               const uint16_t* q_gate, const uint16_t* k, const uint16_t* v,
                               float* out);
size_t gqa_prefill_ws_bytes(int batch, int T);
cudaError_t launch_dn_prefill(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                              const uint16_t* qkv, const float* a, const float* b, float* y,
                              const float* z, float* out);
size_t dn_prefill_ws_bytes(int batch, int T);

// Raises a kernel's dynamic shared memory limit once per device.  `done` holds
// one bit per device and is atomic: contexts on different devices (and the
// allocation-free entry point) may be driven from different host threads.
// Setting the attribute twice is harmless, so a lost race only repeats it.
template <typename Kernel>
cudaError_t set_smem_once(std::atomic<uint64_t>& done, int device, Kernel kern, int bytes) {
    const uint64_t bit = (device >= 0 && device < 64) ? (1ull << device) : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace qm

#define QM_CHECK_CUDA(ctx, expr)                                  \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return qm::cuda_error(ctx, _e, #expr); \
    } while (0)
