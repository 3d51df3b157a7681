/*
 * qora_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the QORA-4B reference's f32 token-mixer path (Rust,
 * src/gemv.rs + src/simd.rs + src/convert.rs of qora-protocol/QORA-LLM-4B).
 * It is the parity checker for the CUDA kernels and the timed CPU baseline
 * ("kind": "port").  Nothing in the product library links or calls it.
 *
 * PARITY UNPINNED: the reference ships no tests, no golden vectors and no
 * fixtures, and it cannot be built here (no Rust toolchain), so this
 * restatement cannot be checked against the reference's own outputs.  It is
 * anchored instead by analytic known-answer cases, by an independent float64
 * restatement in the test suite, and by scalar-vs-AVX-512 agreement.
 *
 * Every function states the reference lines it follows.  Arithmetic follows
 * the Rust code statement by statement: f32 throughout, sequential sums,
 * no fused multiply-add except where the reference itself calls
 * _mm512_fmadd_ps (the file is compiled with -ffp-contract=off).
 */
#ifndef QORA_ORACLE_H
#define QORA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mixer shape fields of Qor4bConfig (src/config.rs:4-32, default_4b 42-79). */
typedef struct or_cfg {
    int num_qk_heads;      /* 16  */
    int num_v_heads;       /* 32  */
    int dn_head_dim;       /* 128 */
    int conv_kernel;       /* 4   */
    int num_attn_heads;    /* 16  */
    int num_kv_heads;      /* 4   */
    int attn_head_dim;     /* 256 */
    int rope_dim;          /* 64 = attn_head_dim * 0.25 (config.rs:82-84) */
} or_cfg;

void or_cfg_default_4b(or_cfg* c);

/* src/simd.rs:18-27 has_avx512 */
int or_has_avx512(void);

/* src/convert.rs:161-176: partial-RoPE tables, [max_pos, rope_dim/2] f32. */
void or_rope_table(float theta, int rope_dim, int max_pos, float* cos_t, float* sin_t);

/*
 * src/gemv.rs:744-883 — the DeltaNet mixer region of forward_deltanet_decode
 * for ONE token of ONE sequence.  qkv = in_proj_qkv output [qkv_dim];
 * a, b = in_proj_a/b outputs [num_v]; state s [num_v, hd, hd] (row = v-dim),
 * conv_buf [qkv_dim, ks-1], *conv_pos.  y [num_v*hd] receives the raw
 * per-head outputs (gemv.rs:814-862).  If z != NULL the epilogue 864-883 is
 * run and gated [num_v*hd] receives y_normed * silu(z).
 * use_avx512 selects simd.rs:292-362 (only when compiled with AVX-512).
 */
void or_dn_decode(const or_cfg* c, const float* qkv, const float* a, const float* b,
                  const float* conv_w, const float* a_log, const float* dt_bias,
                  float* s, float* conv_buf, int64_t* conv_pos, int use_avx512,
                  float* y, const float* z, const float* norm_gamma, float* gated);

/*
 * src/gemv.rs:1119-1219 — the sequential loop of prefill_deltanet_layer for
 * T tokens of ONE sequence.  qkv is given either as f32 (qkv_f32) or as
 * bf16 bits (qkv_bf16, widened exactly), [T, qkv_dim].  a, b: [T, num_v].
 * Only V heads in [vh_lo, vh_hi) run the state update (the heads are
 * independent; the conv buffer is updated for every channel as in
 * 1133-1147).  y: [T, num_v*hd] (rows of other heads untouched).
 * If z != NULL, step 4 (1205-1219) is applied in place to y for the heads
 * in range (the reference does it for all heads).
 */
void or_dn_prefill(const or_cfg* c, int T, const float* qkv_f32, const uint16_t* qkv_bf16,
                   const float* a, const float* b,
                   const float* conv_w, const float* a_log, const float* dt_bias,
                   float* s, float* conv_buf, int64_t* conv_pos,
                   int vh_lo, int vh_hi, float* y,
                   const float* z, const float* norm_gamma);

/*
 * src/gemv.rs:927-1011 — the attention region of forward_attn_decode for
 * ONE token of ONE sequence.  q_gate [H*2*D] interleaved per head
 * (Q_h, Gate_h); k_new, v_new [KVH*D]; q_norm/k_norm gamma [D] (applied as
 * 1+gamma); cos/sin tables [max_pos, rope_dim/2].  KV cache k_cache/v_cache
 * in the reference layout [seq, KVH, D] f32 with room for *seq_len + 1
 * rows; the new row is appended and *seq_len incremented (953-955).
 * out [H*D] = gated attention output (1008-1011).  Heads run on an OpenMP
 * pool when the cache holds >= 64 positions, as rayon does (962-983).
 * Returns 0, or -1 if the position is beyond the RoPE table.
 */
int or_gqa_decode(const or_cfg* c, const float* q_gate, const float* k_new, const float* v_new,
                  const float* q_norm, const float* k_norm,
                  const float* cos_t, const float* sin_t, int max_pos,
                  float* k_cache, float* v_cache, int64_t* seq_len, float* out);

/*
 * src/gemv.rs:1364-1444 — the attention region of prefill_attn_layer for
 * ONE sequence of S tokens, evaluated for a chosen set of query rows.
 * q_gate [S, H*2*D], k_in/v_in [S, KVH*D] given as f32 or bf16 bits.
 * k_cache_out/v_cache_out (nullable) receive the cache the reference
 * stores at 1397-1400: [S, KVH, D] f32, K after QK-norm and RoPE, V raw.
 * rows[nrows] lists query rows t1; out [nrows, H*D] receives the gated
 * attention output of each (1406-1444).  Heads run on an OpenMP pool.
 */
int or_gqa_prefill_rows(const or_cfg* c, int S,
                        const float* q_gate_f32, const uint16_t* q_gate_bf16,
                        const float* k_f32, const uint16_t* k_bf16,
                        const float* v_f32, const uint16_t* v_bf16,
                        const float* q_norm, const float* k_norm,
                        const float* cos_t, const float* sin_t, int max_pos,
                        const int* rows, int nrows, float* out,
                        float* k_cache_out, float* v_cache_out);

/* Threads the OpenMP pool uses (omp_get_max_threads, 1 without OpenMP). */
int or_num_threads(void);
void or_set_num_threads(int n);

/* Q4 / F16 weight GEMV of the projections around the mixers (src/gemv.rs:286-300,
 * 338-368, 411-450; format src/convert.rs:437-467). */
void or_quantize_q4(const float* w, int k, int n, uint8_t* packed, uint16_t* scales);
void or_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales, int k, int n, float* y);
void or_gemv_f16(const float* x, const uint16_t* w, int k, int n, float* y);

/* lm_head over tied embedding rows, penalties, sampling */
void or_lm_head_f16(const float* x, const uint16_t* e, int vocab, int hidden, float* y);
void or_lm_head_q4(const float* x, const uint8_t* packed, const uint16_t* scales, int vocab, int hidden,
                   float* y);
void or_repetition_penalty(float* logits, int vocab, const int32_t* gen, int len, float penalty);
void or_presence_penalty(float* logits, int vocab, const int32_t* gen, int len, float penalty);
int or_sample_top_k(const float* logits, int vocab, float temperature, float top_p, int top_k, float r,
                    double* margin);
float or_rng_next_f32(uint64_t* state);

#ifdef __cplusplus
}
#endif
#endif
