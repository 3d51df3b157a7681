/*
 * qora_mixer.h — C ABI of the B200 (sm_100a) QORA-4B token-mixer library.
 *
 * The library replaces the mixer regions of the reference engine
 * (qora-protocol/QORA-LLM-4B, Rust): the Gated-DeltaNet layers and the
 * full-attention GQA layers, for decode and prefill.  Projections, MLP and
 * residual stay with the caller, exactly where the reference keeps them.
 *
 * Conventions
 *  - Every function returns int: QM_OK (0) or a QM_E_* code; nothing aborts
 *    or throws across this boundary.  qm_last_error(ctx) describes the last
 *    failure on that context.
 *  - Tensors passed to the non-_host entry points are DEVICE pointers on
 *    the context's device; _host variants take host pointers (pinned or
 *    pageable), copy in, run, copy out and return after the results are in
 *    host memory, like the reference's Vec<f32>-returning functions.
 *  - A context binds one device and one CUDA stream; calls on it are
 *    asynchronous and must be serialised by the caller (the reference
 *    drives its GPU from one dedicated thread, gpu_inference.rs:946-953).
 *  - A state/cache handle holds B sequences that advance together: one
 *    decode call adds one token to each of the B sequences (a batch of B
 *    reference caches stepped in lockstep).
 *  - Shapes are those of Qor4bConfig::default_4b (src/config.rs:42-79);
 *    qm_shape_get reports them.  Kernels are specialised for them.
 *  - bf16 tensors are passed as uint16_t bit patterns.
 */
#ifndef QORA_MIXER_H
#define QORA_MIXER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* Status codes.  The reference panics on a layer/cache type mismatch   */
/* (src/gemv.rs:1049,228; src/gpu_inference.rs:418); here that is       */
/* QM_E_MISMATCH.                                                       */
/* ------------------------------------------------------------------ */
#define QM_OK 0
#define QM_E_ARG 1          /* null pointer or invalid value             */
#define QM_E_SHAPE 2        /* batch/size/capacity does not fit          */
#define QM_E_OOM 3          /* device allocation failed                  */
#define QM_E_CUDA 4         /* CUDA runtime/driver error                 */
#define QM_E_NCCL 5         /* NCCL error                                */
#define QM_E_TIMEOUT 6      /* a bounded device-side wait gave up        */
#define QM_E_RANGE 7        /* position beyond the RoPE table or cache   */
#define QM_E_MISMATCH 8     /* handle belongs to another ctx / wrong kind*/
#define QM_E_UNSUPPORTED 9  /* device is not sm_100 (B200)               */
#define QM_E_CAPTURE 10     /* would allocate during CUDA-graph capture  */

typedef struct qm_ctx qm_ctx;
typedef struct qm_dn_state qm_dn_state;
typedef struct qm_kv qm_kv;

/* Mixer shape (fields of Qor4bConfig used by the mixers, src/config.rs:4-32). */
typedef struct qm_shape {
    int num_qk_heads;    /* 16 */
    int num_v_heads;     /* 32 */
    int dn_head_dim;     /* 128 */
    int conv_kernel;     /* 4 */
    int num_attn_heads;  /* 16 */
    int num_kv_heads;    /* 4 */
    int attn_head_dim;   /* 256 */
    int rope_dim;        /* 64 (config.rs:82-84) */
    float rope_theta;    /* 1e7 */
    float rms_eps;       /* 1e-6 */
} qm_shape;

/* How the library was built (no reference counterpart): a bit set of
 * QM_BUILD_* flags.  QM_BUILD_BOUNDS_CHECKS: the checked build
 * (libqora_mixer_checked.so, -DQM_CHECK_BOUNDS), whose prefill and GEMM
 * kernels compare their computed buffer offsets with the buffers' extents
 * and, instead of an out-of-range access, skip it and set the error word
 * (qm_sync then returns QM_E_RANGE). */
#define QM_BUILD_BOUNDS_CHECKS 1
int qm_build_flags(void);

/* Replaces Qor4bConfig::default_4b (src/config.rs:42-79) for the mixer fields. */
int qm_shape_get(qm_shape* out);
const char* qm_status_string(int status);

/* ------------------------------------------------------------------ */
/* Context                                                              */
/* ------------------------------------------------------------------ */
/* Replaces the backend/device set-up of generate_gpu_inner
 * (src/gpu_inference.rs:981-1004).  Fails with QM_E_UNSUPPORTED unless the
 * device is compute capability 10.x. */
int qm_ctx_create(int device, qm_ctx** out);
int qm_ctx_destroy(qm_ctx* ctx);
/* Run subsequent calls on `stream` (a cudaStream_t, taken verbatim: NULL is
 * the legacy default stream).  A new context starts on a stream of its own,
 * which qm_ctx_get_stream returns. */
int qm_ctx_set_stream(qm_ctx* ctx, void* stream);
void* qm_ctx_get_stream(const qm_ctx* ctx);
/* Waits for the context's stream, then reports any device-side error word
 * (a bounded wait that gave up) as QM_E_TIMEOUT. */
int qm_sync(qm_ctx* ctx);
const char* qm_last_error(const qm_ctx* ctx);
/* Grows the context workspace to `bytes` now, so later calls never
 * allocate (needed before capturing calls into a CUDA graph). */
int qm_ctx_reserve(qm_ctx* ctx, size_t bytes);
/* Number of overlapped parts the _host variants cut a batch into (part i's
 * input copy, kernels and output copy run on three streams, so neighbouring
 * parts overlap): dn_parts for qm_dn_decode_host, gqa_parts for
 * qm_gqa_decode_host, 1..8, or 0 for the default (2 from batch 8 up). */
int qm_ctx_set_host_parts(qm_ctx* ctx, int dn_parts, int gqa_parts);
/* on != 0 (the default): when a _host call's buffers are page-locked host
 * memory mapped into the device's address space (cudaHostAlloc,
 * cudaHostRegister, a pinned torch tensor), each range inside its
 * allocation, the kernels use them in place, reading inputs and writing
 * outputs over PCIe, no staging copies and one synchronisation at the end
 * (every buffer of the call must be mapped).  Otherwise (pageable memory)
 * a call is staged through overlapped copies.
 * on == 0 stages every call.  qm_ctx_host_calls counts the calls that took
 * each path. */
int qm_ctx_set_host_direct(qm_ctx* ctx, int on);
int qm_ctx_host_calls(const qm_ctx* ctx, int64_t* in_place, int64_t* staged);
/* Kernels this context launched since creation (for launch accounting). */
int64_t qm_ctx_launch_count(const qm_ctx* ctx);
/* Per-kernel timing: when on, every launch is bracketed by CUDA events on the
 * context stream.  qm_ctx_kernel_time waits for the recorded events and
 * returns the summed device time (ms) and launch count of kernel `name`
 * ("dn_decode", "gqa_prep", "gqa_attn", "gqa_combine", "gqa_prefill",
 * "dn_prefill", ...).  qm_ctx_set_timing(ctx, 0) discards the records. */
int qm_ctx_set_timing(qm_ctx* ctx, int on);
int qm_ctx_kernel_time(qm_ctx* ctx, const char* name, double* total_ms, int64_t* launches);

/* ------------------------------------------------------------------ */
/* RoPE tables                                                           */
/* ------------------------------------------------------------------ */
/* Replaces the table precompute of src/convert.rs:161-176 (loaded at
 * src/save.rs:345-346, uploaded at src/gpu_loader.rs:174-184), with the
 * same f32 formula, for any max_pos (the reference stops at 8192).
 * Host buffers [max_pos, rope_dim/2]. */
int qm_rope_table(float theta, int rope_dim, int max_pos, float* cos_host, float* sin_host);

/* ------------------------------------------------------------------ */
/* DeltaNet recurrent state                                              */
/* ------------------------------------------------------------------ */
/* Replaces DeltaNetState::new (src/gemv.rs:144-157) / GpuDeltaNetState
 * (src/gpu_inference.rs:30-36,49-58) for B sequences: S [B,32,128,128] f32
 * (row = v-dim, as the reference stores it), the causal-conv history and
 * conv_pos, all zero. */
int qm_dn_state_create(qm_ctx* ctx, int batch, qm_dn_state** out);
/* Handles may outlive their context only to be destroyed; destroy frees the
 * storage on the handle's device without touching the context. */
/* Same over caller-owned device memory (not freed by destroy):
 * s [B,32,128,128] f32 and conv [B,4,8192] f32 (see qm_dn_state_data). */
int qm_dn_state_wrap(qm_ctx* ctx, int batch, float* s, float* conv, qm_dn_state** out);
int qm_dn_state_destroy(qm_dn_state* st);
/* Zero S, the conv history and conv_pos (DeltaNetState::new). */
int qm_dn_state_reset(qm_ctx* ctx, qm_dn_state* st);
/* Deep copy (HybridCache::snapshot, src/gemv.rs:198-212). */
int qm_dn_state_snapshot(qm_ctx* ctx, const qm_dn_state* src, qm_dn_state** out);
/* Copy src into dst (HybridCache::restore_from, src/gemv.rs:215-231);
 * QM_E_MISMATCH when the batch sizes differ. */
int qm_dn_state_restore(qm_ctx* ctx, qm_dn_state* dst, const qm_dn_state* src);
/* Sequence b of the state in the reference layout (synchronous):
 * s [32,128,128] and conv_buf [8192,3] (oldest first, gemv.rs:137-139). */
int qm_dn_state_read(qm_ctx* ctx, const qm_dn_state* st, int b, float* s_host, float* conv_buf_host);
int qm_dn_state_write(qm_ctx* ctx, qm_dn_state* st, int b, const float* s_host, const float* conv_buf_host);
int64_t qm_dn_state_conv_pos(const qm_dn_state* st);
int qm_dn_state_set_conv_pos(qm_dn_state* st, int64_t conv_pos);
int qm_dn_state_batch(const qm_dn_state* st);
/* Raw device storage: S [B,32,128,128] f32; conv history [B,4,8192] f32 as a
 * ring of 4 slots, token t stored in slot t % 4. */
int qm_dn_state_data(const qm_dn_state* st, float** s, float** conv);

/* DeltaNet layer parameters (device pointers). */
typedef struct qm_dn_params {
    const float* conv_w;     /* [8192, 4] conv1d_weight (gemv.rs:68)        */
    const float* a_log;      /* [32]  A_log (gemv.rs:69)                    */
    const float* dt_bias;    /* [32]  dt_bias (gemv.rs:70)                  */
    const float* norm_gamma; /* [128] attn_norm_weight widened from f16
                                (gemv.rs:71); only read when z != NULL      */
} qm_dn_params;

/*
 * DeltaNet decode, one token per sequence.  Replaces the mixer region
 * src/gemv.rs:744-883 of forward_deltanet_decode (gemv.rs:719) and
 * src/gpu_inference.rs:149-227 of forward_deltanet_decode_gpu (125):
 * causal conv1d + SiLU, per-head L2 norm (q scaled by 1/sqrt(128)),
 * alpha/beta gates, the gated delta-rule update of S and y = S q.
 *   qkv [B,8192] f32  in_proj_qkv output (Q 0..2047, K 2048..4095, V 4096..)
 *   a,b [B,32]   f32  in_proj_a / in_proj_b outputs
 *   y   [B,32,128] f32 raw per-head output (gemv.rs:814-862); may be NULL
 *       when out is given
 *   z   [B,4096] f32 or NULL: in_proj_z output; when given, out [B,4096]
 *       receives RMSNorm(y)*gamma*SiLU(z) (gemv.rs:864-883), the input of
 *       out_proj.
 */
int qm_dn_decode(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                 const float* a, const float* b, float* y, const float* z, float* out);
/* Host-buffer variant of qm_dn_decode (params stay device pointers). */
int qm_dn_decode_host(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                      const float* a, const float* b, float* y, const float* z, float* out);

/*
 * T sequential DeltaNet decode steps per sequence in one launch: the same
 * result as T qm_dn_decode calls, with the f32 state kept on chip for the
 * whole call (one read and one write of S instead of one per token).
 * Replaces the per-token loop of prefill_deltanet_layer
 * (src/gemv.rs:1129-1203) and T successive mixer regions of
 * forward_deltanet_decode (src/gemv.rs:744-883) when the inputs are known
 * ahead (a prompt, a draft to verify).  f32 arithmetic throughout, so the
 * decode tolerance applies, unlike the tensor-core qm_dn_prefill.
 *   qkv [B,T,8192] f32 (16-byte aligned), a,b [B,T,32] f32,
 *   y [B,T,nvh,128] f32 or NULL when out is given,
 *   z [B,T,4096] f32 or NULL; when given, out [B,T,nvh,128] receives
 *   RMSNorm(y)*gamma*SiLU(z) per token.
 * Works on head-sharded states like qm_dn_decode.
 */
int qm_dn_decode_seq(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T, const float* qkv,
                     const float* a, const float* b, float* y, const float* z, float* out);

/*
 * DeltaNet prefill of T tokens per sequence (chunked WY form on the tensor
 * cores).  Replaces the sequential loop src/gemv.rs:1119-1219 of
 * prefill_deltanet_layer (1086) and the CPU recurrence that
 * prefill_deltanet_layer_gpu runs between device round trips
 * (src/gpu_inference.rs:464-604).
 *   qkv [B,T,8192] bf16, a,b [B,T,32] f32, y [B,T,32,128] f32 (required),
 *   z [B,T,4096] f32 or NULL; when given, out [B,T,4096] f32 receives
 *   RMSNorm(y)*gamma*SiLU(z) (gemv.rs:1205-1219).
 * The state continues from its current contents (conv history included).
 * Chunks of 64 tokens; intra-chunk products are compensated fp16 tcgen05
 * MMAs (hi.hi + hi.lo + lo.hi), the 64x64 triangular solve is f32.
 */
int qm_dn_prefill(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T, const uint16_t* qkv,
                  const float* a, const float* b, float* y, const float* z, float* out);

/* Host-buffer variant of qm_dn_prefill (params stay device pointers):
 * qkv, a, b, y, z, out are host memory (pinned or pageable).  The inputs
 * are copied into the context's staging buffer, the prefill runs, and y
 * (and out) are copied back before the call returns — the reference's GPU
 * prefill flow, which moves each layer's activations down and up around its
 * recurrence (src/gpu_inference.rs:464-476, 591-604). */
int qm_dn_prefill_host(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                       const uint16_t* qkv, const float* a, const float* b, float* y, const float* z,
                       float* out);

/* Head-sharded state (multi-GPU, see qm_shard_plan): V heads
 * [vh_lo, vh_lo + nvh) of every sequence, S [B,nvh,128,128]; vh_lo and nvh
 * even (V heads 2j and 2j+1 share QK head j, gemv.rs:803-809, whose conv
 * history the shard advances).  Decode on such a state reads the full-width
 * inputs (qkv [B,8192], a/b [B,32], z [B,4096]) and writes y [B,nvh,128]
 * and out [B,nvh*128] for its heads only.  Prefill takes full states only
 * (QM_E_UNSUPPORTED).  qm_dn_state_create/wrap are the full range [0,32). */
int qm_dn_state_create_heads(qm_ctx* ctx, int batch, int vh_lo, int nvh, qm_dn_state** out);
int qm_dn_state_wrap_heads(qm_ctx* ctx, int batch, int vh_lo, int nvh, float* s, float* conv,
                           qm_dn_state** out);
int qm_dn_state_heads(const qm_dn_state* st, int* vh_lo, int* nvh);
/* ------------------------------------------------------------------ */
/* GQA KV cache                                                          */
/* ------------------------------------------------------------------ */
/* Replaces KvCacheEntry (src/gemv.rs:164-168, f32 [seq,4,256] grown per
 * token) and GpuKvCacheEntry (src/gpu_inference.rs:38-42, re-concatenated
 * every token, 303-310) with a preallocated bf16 cache
 * K,V [B,4,capacity,256], appended in place. */
int qm_kv_create(qm_ctx* ctx, int batch, int capacity, qm_kv** out);
/* Same over caller-owned device memory k, v (bf16 [B,4,capacity,256]). */
int qm_kv_wrap(qm_ctx* ctx, int batch, int capacity, uint16_t* k, uint16_t* v, qm_kv** out);
int qm_kv_destroy(qm_kv* kv);
int qm_kv_snapshot(qm_ctx* ctx, const qm_kv* src, qm_kv** out);    /* gemv.rs:198-212 */
int qm_kv_restore(qm_ctx* ctx, qm_kv* dst, const qm_kv* src);      /* gemv.rs:215-231 */
int64_t qm_kv_seq_len(const qm_kv* kv);
/* Declare how many positions the cache holds (after filling it directly). */
int qm_kv_set_seq_len(qm_kv* kv, int64_t seq_len);
int qm_kv_capacity(const qm_kv* kv);
int qm_kv_batch(const qm_kv* kv);
int qm_kv_data(const qm_kv* kv, uint16_t** k, uint16_t** v);

/* Head-sharded cache: KV heads [kv_lo, kv_lo + nkv), K,V [B,nkv,capacity,256].
 * Decode on it reads the full-width q_gate [B,16,512] and k_new/v_new
 * [B,4,256] and writes out [B,nkv*4,256] (the query heads of its KV heads).
 * Prefill takes full caches only (QM_E_UNSUPPORTED). */
int qm_kv_create_heads(qm_ctx* ctx, int batch, int capacity, int kv_lo, int nkv, qm_kv** out);
int qm_kv_wrap_heads(qm_ctx* ctx, int batch, int capacity, int kv_lo, int nkv, uint16_t* k,
                     uint16_t* v, qm_kv** out);
int qm_kv_heads(const qm_kv* kv, int* kv_lo, int* nkv);
/* GQA layer parameters (device pointers). */
typedef struct qm_gqa_params {
    const float* q_norm;   /* [256] q_norm widened from f16, applied as 1+g (gemv.rs:86,594) */
    const float* k_norm;   /* [256] k_norm, same                                          */
    const float* rope_cos; /* [max_pos, 32] (convert.rs:165-172)                          */
    const float* rope_sin; /* [max_pos, 32]                                               */
    int max_pos;
} qm_gqa_params;

/*
 * GQA decode, one token per sequence.  Replaces the attention region
 * src/gemv.rs:927-1011 of forward_attn_decode (907) and
 * src/gpu_inference.rs:269-349 of forward_attn_decode_gpu (247):
 * QK-RMSNorm (1+gamma), partial RoPE at position seq_len, KV append,
 * softmax(q K^T / 16) V over seq_len+1 positions, sigmoid output gate.
 *   q_gate [B,16,512] f32 q_proj output, per head Q then gate (gemv.rs:927)
 *   k_new, v_new [B,4,256] f32 k_proj / v_proj outputs
 *   out [B,16,256] f32 gated attention output (input of o_proj)
 * QM_E_RANGE if seq_len >= capacity or seq_len >= max_pos.
 * Uses the context workspace for split-KV partials (grown on first use).
 * Cache rows at and past seq_len are never used, whatever they hold.
 * The kernels run under programmatic dependent launch: the layer parameters
 * (q_norm, k_norm, the RoPE rows) and the cache rows below seq_len - 1 may be
 * read before they wait for the preceding kernel of the stream, q_gate,
 * k_new, v_new and cache row seq_len - 1 only after it; so the kernel just
 * before a call may write the call's inputs and append row seq_len - 1, not
 * the parameters or older rows.
 */
int qm_gqa_decode(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, const float* q_gate,
                  const float* k_new, const float* v_new, float* out);
int qm_gqa_decode_host(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, const float* q_gate,
                       const float* k_new, const float* v_new, float* out);

/*
 * GQA causal prefill of T tokens per sequence.  Replaces the attention
 * region src/gemv.rs:1364-1444 of prefill_attn_layer (1339) and
 * src/gpu_inference.rs:690-766 (which materialises [16,S,S] scores).
 * Like the reference (gemv.rs:1397-1400) it REPLACES the cache contents:
 * positions 0..T-1 receive K after QK-norm + RoPE and raw V (bf16), and
 * seq_len becomes T.
 *   q_gate [B,T,16,512] bf16, k, v [B,T,4,256] bf16, out [B,T,16,256] f32.
 */
int qm_gqa_prefill(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, int T, const uint16_t* q_gate,
                   const uint16_t* k, const uint16_t* v, float* out);

/* Host-buffer variant of qm_gqa_prefill: q_gate, k, v, out in host memory
 * (the reference's prefill_attn_layer_gpu uploads its activations and reads
 * the output back, src/gpu_inference.rs:690-766); returns after out is in
 * host memory. */
int qm_gqa_prefill_host(qm_ctx* ctx, const qm_gqa_params* p, qm_kv* kv, int T, const uint16_t* q_gate,
                        const uint16_t* k, const uint16_t* v, float* out);

/* ------------------------------------------------------------------ */
/* GQA decode without any device allocation                             */
/* ------------------------------------------------------------------ */
/* Size of the library's fixed device scratch array for the entry point
 * below: 16 MiB, held on every GPU that loads the library until exit. */
#define QM_NOALLOC_SCRATCH_BYTES (16u << 20)

/*
 * qm_gqa_decode_noalloc — no counterpart in the reference (it adds a way to
 * call the GQA decode kernels, not a reference function).
 *
 * Same computation as qm_gqa_decode, for callers that cannot call
 * cudaMalloc: a serving engine whose memory manager reserves all device
 * memory up front and forbids later allocations, or a plugin that only
 * borrows its host's buffers and stream.  Such callers cannot create a
 * qm_ctx, which allocates.  The caller passes everything by pointer:
 *   k_cache, v_cache  bf16 [batch,4,capacity,256] (16-byte aligned)
 *   seq_len           cached positions; the new token is written at index
 *                     seq_len and the caller advances its own count
 *   q_gate, k_new, v_new, out  as in qm_gqa_decode
 *   stream            cudaStream_t on the current device (NULL = legacy)
 * The split-KV partials go to a fixed device array inside the library
 * (QM_NOALLOC_SCRATCH_BYTES per GPU).  Nothing is allocated: no cudaMalloc,
 * cudaFree or allocating library call.  A request whose partials do not fit
 * returns QM_E_SHAPE: they take about 36 KB per sequence plus 16.5 KB per
 * (sequence, KV split); on a 148-SM B200, batch 16 fits at 32K context and
 * batch 64 does not.
 * The first call on each device does a one-time set-up with that device
 * current (looks up the array's device address, reads the SM count); make
 * that first call before any stream capture.  Every call on a device shares
 * the one array and it keeps the last call's contents, so calls that
 * overlap on the GPU (different streams, or other host threads) race:
 * serialise them.  Returns after enqueueing the work; device-side wait
 * timeouts are not reported by this entry point.
 */
int qm_gqa_decode_noalloc(const qm_gqa_params* p, uint16_t* k_cache, uint16_t* v_cache, int batch,
                          int capacity, int64_t seq_len, const float* q_gate, const float* k_new,
                          const float* v_new, float* out, void* stream);

/* ------------------------------------------------------------------ */
/* Projections around the mixers (the next component beside the path):  */
/* y[b] = x[b] . W for the reference's weight formats                    */
/* (src/gemv.rs:21-40, gemv 286-300): W [k rows (input) x n (output)].   */
/* ------------------------------------------------------------------ */
#define QM_W_F16 0  /* data: f16 [k][n] (gemv_f16, src/gemv.rs:338-368)           */
#define QM_W_Q4 1   /* data: uint8 [k][n/2], even column in the low nibble, value */
                    /* q - 8; scales: f16 [k][n/32] (gemv_q4, src/gemv.rs:411-450; */
                    /* format src/convert.rs:437-467)                             */
#define QM_W_F16_ROWS 2  /* one row per output, f16 [n][k]: the tied embedding as */
                         /* lm_head (src/gemv.rs:664-676)                         */
#define QM_W_Q4_ROWS 3   /* one row per output, packed [n][k/2] and f16 scales    */
                         /* [n][k/32], groups of 32 along k (src/gemv.rs:677-707) */
typedef struct qm_weight {
    int kind;            /* QM_W_F16 or QM_W_Q4 */
    int k, n;
    const void* data;    /* device */
    const void* scales;  /* device, Q4 only */
} qm_weight;
/* y[batch][n] = x[batch][k] . W on the context's stream (device pointers);
 * replaces gemv(input, weight) (src/gemv.rs:286-291) at decode batch sizes.
 * Q4 needs n % 32 == 0, F16 n % 8 == 0.  Sums are f32 and added in a fixed
 * order (the result does not depend on timing).  The kernel issues its
 * weight loads before it waits for the preceding kernel of the stream
 * (programmatic dependent launch): it reads x only after that kernel is done.
 * Calls on one context share a scratch area (partial sums, allocated by the
 * first call that needs it; QM_E_CAPTURE if that call is inside a stream
 * capture): issue them in order on the context's stream. */
int qm_gemv(qm_ctx* ctx, const qm_weight* w, int batch, const float* x, float* y);
/* ys[i][batch][ws[i].n] = x[batch][k] . W_i for count <= 4 weights of one
 * kind and one k that share the input, in one launch: the reference's
 * in_proj_qkv / a / b / z of one x_norm (src/gemv.rs:742,788-789,865) or
 * q / k / v_proj (src/gemv.rs:928,941-942).  QM_E_MISMATCH when the weights
 * differ in k or kind.  ys is a host array of device pointers. */
int qm_gemv_multi(qm_ctx* ctx, const qm_weight* ws, int count, int batch, const float* x,
                  float* const* ys);
/* y[T][n] = x[T][k] . W for a whole prompt on the tensor cores: the
 * reference's gemm over seq_len tokens (src/gemv.rs:294-300, its prefill at
 * 1114-1117, 1222, 1366-1385), for both weight formats it dispatches on
 * (gemm_q4 / gemm_f16, src/gemv.rs:390, 529): QM_W_Q4 [k][n/2] or QM_W_F16
 * [k][n] (data 16-byte aligned), or their row layouts QM_W_Q4_ROWS /
 * QM_W_F16_ROWS (the tied embedding as a batched lm_head, src/gemv.rs:677-707);
 * k % 64 == 0, n % 32 == 0;
 * x bf16 [T][k] (16-byte aligned, as the prefill mixers take their inputs),
 * y f32 [T][n].  The weights are rounded to bf16 on the way in (Q4: the
 * scale, then the product):
 * max|y - exact| / RMS(y) is a few 1e-3.  When T and n give fewer 256 x 256
 * tiles than half the SMs, K is split over up to 4 CTAs a tile whose partial
 * sums meet in the scratch area qm_gemv uses (same rules: a fixed order of
 * addition, QM_E_CAPTURE if it must grow inside a stream capture). */
int qm_gemm(qm_ctx* ctx, const qm_weight* w, int T, const uint16_t* x, float* y);
/* The same with y bf16 [T][n] (the f32 sum rounded to nearest): the form the
 * prefill mixers take their q / k / v in (qm_dn_prefill, qm_gqa_prefill). */
int qm_gemm_bf16(qm_ctx* ctx, const qm_weight* w, int T, const uint16_t* x, uint16_t* y);
/* (Row-layout weights, QM_W_F16_ROWS / QM_W_Q4_ROWS, go through qm_gemv with
 * one weight per call: logits[b][v] = x[b] . E[v], the reference's
 * lm_head_parallel, src/gemv.rs:662-711.  Q4 rows need k % 32 == 0.) */

/* ------------------------------------------------------------------ */
/* The decode loop's tail (src/generate.rs:185-198), device pointers.  */
/* ------------------------------------------------------------------ */
/* Penalties on logits[batch][vocab] in the reference's order: repetition
 * (src/generate.rs:58-69: over the last min(len, 64) tokens of each
 * history, every occurrence divides a positive logit by the penalty or
 * multiplies a non-positive one; off when <= 1), presence (72-83: every
 * token of the history loses the penalty once; off when <= 0), then
 * ban_token (>= 0) set to -inf (the EOS ban inside a think block, 191).
 * Sequence b's history is tokens[b * stride + i], i < lens[b]. */
int qm_logits_penalize(qm_ctx* ctx, float* logits, int batch, int vocab, const int* tokens,
                       const int* lens, int stride, float repetition_penalty,
                       float presence_penalty, int ban_token);
/* sample_token_top_k (src/generate.rs:334-384) for each sequence:
 * temperature <= 0 gives the first index of the largest logit; otherwise
 * the top_k largest (value descending, index ascending), softmax at the
 * temperature against the largest logit, the top-p nucleus, and the draw
 * r[b] in [0, 1) (the reference's rng.next_f32(); the caller keeps the
 * generator).  ids[b] receives the token.  top_k must resolve to at most
 * 4096 candidates (QM_E_UNSUPPORTED otherwise; top_k 0 means the whole
 * vocabulary).  Logits must not be NaN (the reference's order is then
 * unspecified). */
int qm_sample(qm_ctx* ctx, const float* logits, int batch, int vocab, float temperature,
              float top_p, int top_k, const float* r, int* ids);

/* ------------------------------------------------------------------ */
/* Multi-GPU (one process per GPU).  The reference runs one device        */
/* (src/gpu_inference.rs:981-1004); these calls spread a decode batch     */
/* over the GPUs of one node.                                             */
/* ------------------------------------------------------------------ */
/* Head-sharded layout of rank `rank` of `world` (1, 2, 4, 8 or 16):
 * DeltaNet V heads [vh_lo, vh_lo+nvh) = 32/world heads per rank; GQA KV
 * heads [kv_lo, kv_lo+nkv) in min(world,4) groups, and, with more than 4
 * ranks, part seq_part of seq_parts equal parts of the batch.  Sequence
 * sharding (whole states per rank) needs no plan and no communication. */
typedef struct qm_shard {
    int world, rank;
    int vh_lo, nvh;
    int kv_lo, nkv;
    int seq_part, seq_parts;
} qm_shard;
int qm_shard_plan(int world, int rank, qm_shard* out);

/* NCCL communicator for the one collective of the head-sharded layout: the
 * all-gather of the per-layer mixer outputs.  libnccl.so.2 is loaded at run
 * time (QM_E_NCCL when absent).  One rank calls qm_comm_unique_id and
 * passes the bytes to the others; every rank then calls qm_comm_create.
 * Calls wait for NCCL at most timeout_ms on the host and then abort the
 * communicator (QM_E_TIMEOUT), so a rank that never joins cannot hang the
 * others. */
#define QM_COMM_ID_BYTES 128
typedef struct qm_comm qm_comm;
int qm_comm_unique_id(unsigned char* id /* [QM_COMM_ID_BYTES] */);
int qm_comm_create(qm_ctx* ctx, const unsigned char* id, int world, int rank, int timeout_ms,
                   qm_comm** out);
/* recv[world * bytes_per_rank] = every rank's send[bytes_per_rank], in rank
 * order, on the context's stream. */
int qm_comm_allgather(qm_comm* comm, const void* send, void* recv, size_t bytes_per_rank);
/* Switches qm_comm_allgather to a peer-memory path for calls of at most
 * max_bytes_per_rank bytes per rank: one kernel stores this rank's bytes
 * straight into every other rank's gather area over NVLink (the areas are
 * mapped once, here, through CUDA IPC) and copies the rows that arrived
 * into recv, with no NCCL kernel and no host wait per call.  Collective:
 * every rank calls it at the same point.  Returns QM_E_UNSUPPORTED on every
 * rank when some rank cannot map another's memory or two ranks share a
 * GPU; NCCL then stays in use.  A device-side wait for a peer gives up
 * after wait_ms and sets the context's error word (qm_sync: QM_E_TIMEOUT);
 * later calls then fail with QM_E_TIMEOUT, as the ranks are out of step.
 * With the peer path on, qm_comm_destroy is collective too: a rank frees
 * its area only after every rank has unmapped it. */
int qm_comm_enable_peer(qm_comm* comm, size_t max_bytes_per_rank, int wait_ms);
int qm_comm_destroy(qm_comm* comm);

#ifdef __cplusplus
}
#endif
#endif /* QORA_MIXER_H */
