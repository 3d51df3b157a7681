/*
 * qora_oracle.c — TEST INFRASTRUCTURE ONLY (parity checker + CPU baseline).
 *
 * C restatement of the QORA-4B reference's CPU f32 token-mixer path.
 * PARITY UNPINNED: the reference has no tests or golden vectors and cannot
 * be built here (Rust is not installed); see qora_oracle.h.
 *
 * Citations are path:line inside the reference project
 * (qora-protocol/QORA-LLM-4B).  Compile with -ffp-contract=off so that
 * a*b+c stays two roundings, as rustc emits it.
 */
#include "qora_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__x86_64__)
#include <immintrin.h>
#include <cpuid.h>
#endif

void or_cfg_default_4b(or_cfg* c) {
    /* src/config.rs:52-78 */
    c->num_qk_heads = 16;
    c->num_v_heads = 32;
    c->dn_head_dim = 128;
    c->conv_kernel = 4;
    c->num_attn_heads = 16;
    c->num_kv_heads = 4;
    c->attn_head_dim = 256;
    /* config.rs:82-84: (256 as f32 * 0.25) as usize */
    c->rope_dim = (int)((float)c->attn_head_dim * 0.25f);
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ---------------------------------------------------------------------- */
/* Shared helpers: src/gemv.rs:569-659                                     */
/* ---------------------------------------------------------------------- */

/* gemv.rs:629-633 */
static inline float silu(float x) { return x / (1.0f + expf(-x)); }

/* gemv.rs:635-639 */
static inline float softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

/* gemv.rs:641-649 */
static void l2_normalize(float* x, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float norm = sqrtf(ss);
    if (norm > 1e-12f) {
        float inv = 1.0f / norm;
        for (int i = 0; i < n; i++) x[i] *= inv;
    }
}

/* gemv.rs:651-659 */
static void softmax_raw(float* s, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, s[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        s[i] = expf(s[i] - mx);
        sum += s[i];
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) s[i] *= inv;
}

/* gemv.rs:583-597: per-head RMSNorm with (1 + gamma), gamma shared over heads */
static void per_head_rms_norm(float* x, int num_heads, int head_dim, const float* gamma) {
    for (int h = 0; h < num_heads; h++) {
        float* head = x + (size_t)h * head_dim;
        float ss = 0.0f;
        for (int d = 0; d < head_dim; d++) ss += head[d] * head[d];
        float inv_rms = 1.0f / sqrtf(ss / (float)head_dim + 1e-6f);
        for (int d = 0; d < head_dim; d++) head[d] = head[d] * inv_rms * (1.0f + gamma[d]);
    }
}

/* gemv.rs:599-627: split-half partial RoPE */
static void apply_partial_rope(float* data, int num_heads, int head_dim, const float* cos_t,
                               const float* sin_t, int rotary_dim, int64_t position) {
    int half = rotary_dim / 2;
    int64_t off = position * half;
    for (int h = 0; h < num_heads; h++) {
        float* base = data + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            float x1 = base[i];
            float x2 = base[half + i];
            float cc = cos_t[off + i];
            float ss = sin_t[off + i];
            base[i] = x1 * cc - x2 * ss;
            base[half + i] = x2 * cc + x1 * ss;
        }
    }
}

/* ---------------------------------------------------------------------- */
/* RoPE table: src/convert.rs:161-176                                      */
/* ---------------------------------------------------------------------- */
void or_rope_table(float theta, int rope_dim, int max_pos, float* cos_t, float* sin_t) {
    int half_dim = rope_dim / 2;
    for (int pos = 0; pos < max_pos; pos++) {
        for (int i = 0; i < half_dim; i++) {
            float freq = 1.0f / powf(theta, 2.0f * (float)i / (float)rope_dim);
            float angle = (float)pos * freq;
            cos_t[(size_t)pos * half_dim + i] = cosf(angle);
            sin_t[(size_t)pos * half_dim + i] = sinf(angle);
        }
    }
}

/* ---------------------------------------------------------------------- */
/* AVX-512 DeltaNet head update: src/simd.rs:292-362 (+ hsum_ps 37-50)     */
/* ---------------------------------------------------------------------- */
int or_has_avx512(void) {
#if defined(__x86_64__)
    /* simd.rs:18-27: is_x86_feature_detected!("avx512f") */
    return __builtin_cpu_supports("avx512f") ? 1 : 0;
#else
    return 0;
#endif
}

#if defined(__x86_64__)
__attribute__((target("avx512f"))) static inline float hsum_ps(__m512 v) {
    __m128 a = _mm512_extractf32x4_ps(v, 0);
    __m128 b = _mm512_extractf32x4_ps(v, 1);
    __m128 c = _mm512_extractf32x4_ps(v, 2);
    __m128 d = _mm512_extractf32x4_ps(v, 3);
    __m128 sum = _mm_add_ps(_mm_add_ps(a, b), _mm_add_ps(c, d));
    __m128 hi = _mm_movehl_ps(sum, sum);
    __m128 sum2 = _mm_add_ps(sum, hi);
    __m128 hi2 = _mm_shuffle_ps(sum2, sum2, 1);
    __m128 sum3 = _mm_add_ss(sum2, hi2);
    return _mm_cvtss_f32(sum3);
}

__attribute__((target("avx512f"))) static void deltanet_head_update_avx512(
    float* state, const float* q, const float* k, const float* v, float alpha, float beta,
    int hd, float* y_out, float* pred /* scratch [hd] */) {
    int hd16 = hd / 16 * 16;
    __m512 al_vec = _mm512_set1_ps(alpha);
    int total = hd * hd;
    for (int i = 0; i < total; i += 16) {
        __m512 s_vec = _mm512_loadu_ps(state + i);
        _mm512_storeu_ps(state + i, _mm512_mul_ps(s_vec, al_vec));
    }
    for (int r = 0; r < hd; r++) {
        const float* row = state + (size_t)r * hd;
        __m512 acc = _mm512_setzero_ps();
        for (int c = 0; c < hd16; c += 16)
            acc = _mm512_fmadd_ps(_mm512_loadu_ps(row + c), _mm512_loadu_ps(k + c), acc);
        pred[r] = hsum_ps(acc);
    }
    for (int r = 0; r < hd; r++) {
        float delta = beta * (v[r] - pred[r]);
        if (delta == 0.0f) continue;
        __m512 dv = _mm512_set1_ps(delta);
        float* row = state + (size_t)r * hd;
        for (int c = 0; c < hd16; c += 16)
            _mm512_storeu_ps(row + c,
                             _mm512_fmadd_ps(dv, _mm512_loadu_ps(k + c), _mm512_loadu_ps(row + c)));
    }
    for (int r = 0; r < hd; r++) {
        const float* row = state + (size_t)r * hd;
        __m512 acc = _mm512_setzero_ps();
        for (int c = 0; c < hd16; c += 16)
            acc = _mm512_fmadd_ps(_mm512_loadu_ps(row + c), _mm512_loadu_ps(q + c), acc);
        y_out[r] = hsum_ps(acc);
    }
}
#endif

/* Scalar head update: src/gemv.rs:836-861 (decode) == 1180-1201 (prefill). */
static void deltanet_head_update_scalar(float* s, const float* q, const float* k, const float* v,
                                        float al, float be, int hd, float* y_out, float* pred) {
    int n = hd * hd;
    for (int i = 0; i < n; i++) s[i] *= al;
    for (int r = 0; r < hd; r++) {
        float dot = 0.0f;
        const float* row = s + (size_t)r * hd;
        for (int c = 0; c < hd; c++) dot += row[c] * k[c];
        pred[r] = dot;
    }
    for (int r = 0; r < hd; r++) {
        float delta = be * (v[r] - pred[r]);
        float* row = s + (size_t)r * hd;
        for (int c = 0; c < hd; c++) row[c] += delta * k[c];
    }
    for (int r = 0; r < hd; r++) {
        float dot = 0.0f;
        const float* row = s + (size_t)r * hd;
        for (int c = 0; c < hd; c++) dot += row[c] * q[c];
        y_out[r] = dot;
    }
}

/* Causal depthwise conv1d + buffer shift: gemv.rs:748-769 == 1132-1147. */
static void conv_step(int qkv_dim, int ks, const float* x, const float* conv_w, float* conv_buf,
                      float* out) {
    int buf_len = ks - 1;
    for (int ch = 0; ch < qkv_dim; ch++) {
        float sum = 0.0f;
        for (int t = 0; t < buf_len; t++)
            sum += conv_buf[(size_t)ch * buf_len + t] * conv_w[(size_t)ch * ks + t];
        sum += x[ch] * conv_w[(size_t)ch * ks + buf_len];
        out[ch] = sum;
    }
    for (int ch = 0; ch < qkv_dim; ch++) {
        float* b = conv_buf + (size_t)ch * buf_len;
        for (int t = 0; t < buf_len - 1; t++) b[t] = b[t + 1];
        b[buf_len - 1] = x[ch];
    }
}

/* ---------------------------------------------------------------------- */
/* DeltaNet decode mixer: src/gemv.rs:744-883                              */
/* ---------------------------------------------------------------------- */
void or_dn_decode(const or_cfg* c, const float* qkv, const float* a, const float* b,
                  const float* conv_w, const float* a_log, const float* dt_bias, float* s,
                  float* conv_buf, int64_t* conv_pos, int use_avx512, float* y, const float* z,
                  const float* norm_gamma, float* gated) {
    const int num_qk = c->num_qk_heads, num_v = c->num_v_heads, hd = c->dn_head_dim;
    const int q_dim = num_qk * hd, k_dim = num_qk * hd, v_dim = num_v * hd;
    const int qkv_dim = q_dim + k_dim + v_dim;
    const int ks = c->conv_kernel;
    const int v_per_qk = num_v / num_qk;
    const float scale = 1.0f / sqrtf((float)hd);

    float* qkv_conv = (float*)malloc(sizeof(float) * qkv_dim);
    float* q_exp = (float*)malloc(sizeof(float) * num_v * hd);
    float* k_exp = (float*)malloc(sizeof(float) * num_v * hd);
    float* alpha = (float*)malloc(sizeof(float) * num_v);
    float* beta = (float*)malloc(sizeof(float) * num_v);
    float* pred = (float*)malloc(sizeof(float) * hd);

    /* 3. conv (744-769) */
    conv_step(qkv_dim, ks, qkv, conv_w, conv_buf, qkv_conv);
    *conv_pos += 1;
    /* 4. SiLU (771-772) */
    for (int i = 0; i < qkv_dim; i++) qkv_conv[i] = silu(qkv_conv[i]);
    /* 5. split + L2 norm + scale (774-785) */
    float* q = qkv_conv;
    float* k = qkv_conv + q_dim;
    const float* v = qkv_conv + q_dim + k_dim;
    for (int h = 0; h < num_qk; h++) {
        l2_normalize(q + (size_t)h * hd, hd);
        l2_normalize(k + (size_t)h * hd, hd);
        for (int j = 0; j < hd; j++) q[(size_t)h * hd + j] *= scale;
    }
    /* 6. alpha, beta (787-800) */
    for (int vh = 0; vh < num_v; vh++) {
        float a_exp = expf(a_log[vh]);
        float sp = softplus(a[vh] + dt_bias[vh]);
        alpha[vh] = expf(-a_exp * sp);
        beta[vh] = 1.0f / (1.0f + expf(-b[vh]));
    }
    /* 7. GVA expansion (802-809) */
    for (int vh = 0; vh < num_v; vh++) {
        int qk_h = vh / v_per_qk;
        memcpy(q_exp + (size_t)vh * hd, q + (size_t)qk_h * hd, sizeof(float) * hd);
        memcpy(k_exp + (size_t)vh * hd, k + (size_t)qk_h * hd, sizeof(float) * hd);
    }
    /* 8. per-head state update (811-862), heads serial (817) */
    int avx = 0;
#if defined(__x86_64__)
    avx = use_avx512 && or_has_avx512();
#endif
    for (int vh = 0; vh < num_v; vh++) {
        float* sh = s + (size_t)vh * hd * hd;
        const float* qh = q_exp + (size_t)vh * hd;
        const float* kh = k_exp + (size_t)vh * hd;
        const float* vv = v + (size_t)vh * hd;
        float* yh = y + (size_t)vh * hd;
#if defined(__x86_64__)
        if (avx) {
            deltanet_head_update_avx512(sh, qh, kh, vv, alpha[vh], beta[vh], hd, yh, pred);
            continue;
        }
#endif
        deltanet_head_update_scalar(sh, qh, kh, vv, alpha[vh], beta[vh], hd, yh, pred);
    }
    /* 9. per-head RMSNorm (plain gamma) * SiLU(z) (864-883) */
    if (z && norm_gamma && gated) {
        for (int h = 0; h < num_v; h++) {
            const float* hs = y + (size_t)h * hd;
            float ss = 0.0f;
            for (int j = 0; j < hd; j++) ss += hs[j] * hs[j];
            float inv_rms = 1.0f / sqrtf(ss / (float)hd + 1e-6f);
            for (int j = 0; j < hd; j++) {
                float yn = hs[j] * inv_rms * norm_gamma[j];
                gated[(size_t)h * hd + j] = yn * silu(z[(size_t)h * hd + j]);
            }
        }
    }
    free(qkv_conv);
    free(q_exp);
    free(k_exp);
    free(alpha);
    free(beta);
    free(pred);
}

/* ---------------------------------------------------------------------- */
/* DeltaNet sequential prefill: src/gemv.rs:1119-1219                      */
/* ---------------------------------------------------------------------- */
void or_dn_prefill(const or_cfg* c, int T, const float* qkv_f32, const uint16_t* qkv_bf16,
                   const float* a, const float* b, const float* conv_w, const float* a_log,
                   const float* dt_bias, float* s, float* conv_buf, int64_t* conv_pos, int vh_lo,
                   int vh_hi, float* y, const float* z, const float* norm_gamma) {
    const int num_qk = c->num_qk_heads, num_v = c->num_v_heads, hd = c->dn_head_dim;
    const int q_dim = num_qk * hd, k_dim = num_qk * hd, v_dim = num_v * hd;
    const int qkv_dim = q_dim + k_dim + v_dim;
    const int ks = c->conv_kernel;
    const int v_per_qk = num_v / num_qk;
    const float scale = 1.0f / sqrtf((float)hd);
    if (vh_lo < 0) vh_lo = 0;
    if (vh_hi > num_v) vh_hi = num_v;

    float* xrow = (float*)malloc(sizeof(float) * qkv_dim);
    float* qkv_conv = (float*)malloc(sizeof(float) * qkv_dim);
    float* q_exp = (float*)malloc(sizeof(float) * num_v * hd);
    float* k_exp = (float*)malloc(sizeof(float) * num_v * hd);
    float* pred = (float*)malloc(sizeof(float) * hd);
    float* a_exp_table = (float*)malloc(sizeof(float) * num_v);
    for (int vh = 0; vh < num_v; vh++) a_exp_table[vh] = expf(a_log[vh]); /* 1127 */

    for (int t = 0; t < T; t++) {
        const float* qkv_t;
        if (qkv_f32) {
            qkv_t = qkv_f32 + (size_t)t * qkv_dim;
        } else {
            const uint16_t* src = qkv_bf16 + (size_t)t * qkv_dim;
            for (int i = 0; i < qkv_dim; i++) xrow[i] = bf16_to_f32(src[i]);
            qkv_t = xrow;
        }
        conv_step(qkv_dim, ks, qkv_t, conv_w, conv_buf, qkv_conv); /* 1132-1146 */
        *conv_pos += 1;                                             /* 1147 */
        for (int i = 0; i < qkv_dim; i++) qkv_conv[i] = silu(qkv_conv[i]); /* 1149 */
        for (int h = 0; h < num_qk; h++) {                                /* 1151-1156 */
            l2_normalize(qkv_conv + (size_t)h * hd, hd);
            l2_normalize(qkv_conv + q_dim + (size_t)h * hd, hd);
            for (int j = 0; j < hd; j++) qkv_conv[(size_t)h * hd + j] *= scale;
        }
        const float* a_t = a + (size_t)t * num_v;
        const float* b_t = b + (size_t)t * num_v;
        for (int vh = 0; vh < num_v; vh++) { /* 1161-1166 */
            int qk_h = vh / v_per_qk;
            memcpy(q_exp + (size_t)vh * hd, qkv_conv + (size_t)qk_h * hd, sizeof(float) * hd);
            memcpy(k_exp + (size_t)vh * hd, qkv_conv + q_dim + (size_t)qk_h * hd,
                   sizeof(float) * hd);
        }
        const float* v_slice = qkv_conv + q_dim + k_dim;
        for (int vh = vh_lo; vh < vh_hi; vh++) { /* 1170-1202 */
            float al = expf(-a_exp_table[vh] * softplus(a_t[vh] + dt_bias[vh]));
            float be = 1.0f / (1.0f + expf(-b_t[vh]));
            deltanet_head_update_scalar(s + (size_t)vh * hd * hd, q_exp + (size_t)vh * hd,
                                        k_exp + (size_t)vh * hd, v_slice + (size_t)vh * hd, al, be,
                                        hd, y + (size_t)t * v_dim + (size_t)vh * hd, pred);
        }
    }
    if (z && norm_gamma) { /* 1205-1219 */
        for (int t = 0; t < T; t++) {
            const float* z_t = z + (size_t)t * v_dim;
            float* y_t = y + (size_t)t * v_dim;
            for (int h = vh_lo; h < vh_hi; h++) {
                float* hs = y_t + (size_t)h * hd;
                float ss = 0.0f;
                for (int j = 0; j < hd; j++) ss += hs[j] * hs[j];
                float inv_rms = 1.0f / sqrtf(ss / (float)hd + 1e-6f);
                for (int j = 0; j < hd; j++) hs[j] = hs[j] * inv_rms * norm_gamma[j];
                for (int j = 0; j < hd; j++) hs[j] *= silu(z_t[(size_t)h * hd + j]);
            }
        }
    }
    free(xrow);
    free(qkv_conv);
    free(q_exp);
    free(k_exp);
    free(pred);
    free(a_exp_table);
}

/* ---------------------------------------------------------------------- */
/* GQA attention for one query vector over positions [0, len):             */
/* src/gemv.rs:964-981 (decode) == 1410-1426 (prefill)                     */
/* ---------------------------------------------------------------------- */
static void attend_one(const float* q_vec, const float* kc, const float* vc, int64_t len,
                       int kv_stride, int kv_off, int head_dim, float scale, float* scores,
                       float* head_out) {
    for (int64_t s = 0; s < len; s++) {
        const float* kr = kc + (size_t)s * kv_stride + kv_off;
        float dot = 0.0f;
        for (int d = 0; d < head_dim; d++) dot += q_vec[d] * kr[d];
        scores[s] = dot * scale;
    }
    softmax_raw(scores, (int)len);
    for (int d = 0; d < head_dim; d++) head_out[d] = 0.0f;
    for (int64_t s = 0; s < len; s++) {
        const float* vr = vc + (size_t)s * kv_stride + kv_off;
        float sc = scores[s];
        for (int d = 0; d < head_dim; d++) head_out[d] += sc * vr[d];
    }
}

/* ---------------------------------------------------------------------- */
/* GQA decode mixer: src/gemv.rs:927-1011                                  */
/* ---------------------------------------------------------------------- */
int or_gqa_decode(const or_cfg* c, const float* q_gate, const float* k_new_in,
                  const float* v_new, const float* q_norm, const float* k_norm,
                  const float* cos_t, const float* sin_t, int max_pos, float* k_cache,
                  float* v_cache, int64_t* seq_len, float* out) {
    const int H = c->num_attn_heads, KVH = c->num_kv_heads, D = c->attn_head_dim;
    const int q_dim = H * D;
    const int groups = H / KVH;
    const int rot = c->rope_dim;
    const int64_t offset = *seq_len;
    if (offset >= max_pos) return -1; /* the reference would index past the table */

    float* q = (float*)malloc(sizeof(float) * q_dim);
    float* gate = (float*)malloc(sizeof(float) * q_dim);
    float* k_new = (float*)malloc(sizeof(float) * KVH * D);
    for (int h = 0; h < H; h++) { /* 932-937 */
        memcpy(q + (size_t)h * D, q_gate + (size_t)h * 2 * D, sizeof(float) * D);
        memcpy(gate + (size_t)h * D, q_gate + (size_t)h * 2 * D + D, sizeof(float) * D);
    }
    memcpy(k_new, k_new_in, sizeof(float) * KVH * D);
    per_head_rms_norm(q, H, D, q_norm);                             /* 945 */
    per_head_rms_norm(k_new, KVH, D, k_norm);                       /* 946 */
    apply_partial_rope(q, H, D, cos_t, sin_t, rot, offset);         /* 949 */
    apply_partial_rope(k_new, KVH, D, cos_t, sin_t, rot, offset);   /* 950 */
    memcpy(k_cache + (size_t)offset * KVH * D, k_new, sizeof(float) * KVH * D); /* 953 */
    memcpy(v_cache + (size_t)offset * KVH * D, v_new, sizeof(float) * KVH * D); /* 954 */
    *seq_len = offset + 1;                                                        /* 955 */
    const int64_t L = *seq_len;
    const float scale = 1.0f / sqrtf((float)D); /* 959 */
    const int kv_stride = KVH * D;

    /* 962-1006: rayon over heads when L >= 64, serial otherwise; per-head
     * arithmetic is identical either way. */
    int par = L >= 64;
#pragma omp parallel for schedule(static) if (par)
    for (int h = 0; h < H; h++) {
        float* scores = (float*)malloc(sizeof(float) * L);
        attend_one(q + (size_t)h * D, k_cache, v_cache, L, kv_stride, (h / groups) * D, D, scale,
                   scores, out + (size_t)h * D);
        free(scores);
    }
    for (int j = 0; j < q_dim; j++) out[j] *= 1.0f / (1.0f + expf(-gate[j])); /* 1009-1011 */
    free(q);
    free(gate);
    free(k_new);
    return 0;
}

/* ---------------------------------------------------------------------- */
/* GQA causal prefill, sampled rows: src/gemv.rs:1364-1444                 */
/* ---------------------------------------------------------------------- */
int or_gqa_prefill_rows(const or_cfg* c, int S, const float* q_gate_f32,
                        const uint16_t* q_gate_bf16, const float* k_f32, const uint16_t* k_bf16,
                        const float* v_f32, const uint16_t* v_bf16, const float* q_norm,
                        const float* k_norm, const float* cos_t, const float* sin_t, int max_pos,
                        const int* rows, int nrows, float* out, float* k_cache_out,
                        float* v_cache_out) {
    const int H = c->num_attn_heads, KVH = c->num_kv_heads, D = c->attn_head_dim;
    const int q_dim = H * D, kv_dim = KVH * D;
    const int groups = H / KVH;
    const int rot = c->rope_dim;
    if (S > max_pos) return -1;
    for (int i = 0; i < nrows; i++)
        if (rows[i] < 0 || rows[i] >= S) return -2;

    /* K: per-token QK-norm + RoPE (1388-1395); V raw (1385). */
    float* k_all = (float*)malloc(sizeof(float) * (size_t)S * kv_dim);
    float* v_all = (float*)malloc(sizeof(float) * (size_t)S * kv_dim);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < S; t++) {
        float* kt = k_all + (size_t)t * kv_dim;
        float* vt = v_all + (size_t)t * kv_dim;
        for (int i = 0; i < kv_dim; i++) {
            size_t idx = (size_t)t * kv_dim + i;
            kt[i] = k_f32 ? k_f32[idx] : bf16_to_f32(k_bf16[idx]);
            vt[i] = v_f32 ? v_f32[idx] : bf16_to_f32(v_bf16[idx]);
        }
        per_head_rms_norm(kt, KVH, D, k_norm);
        apply_partial_rope(kt, KVH, D, cos_t, sin_t, rot, t);
    }
    if (k_cache_out) memcpy(k_cache_out, k_all, sizeof(float) * (size_t)S * kv_dim);
    if (v_cache_out) memcpy(v_cache_out, v_all, sizeof(float) * (size_t)S * kv_dim);

    const float scale = 1.0f / sqrtf((float)D);
    /* Q/gate split (1369-1381), QK-norm + RoPE at position t1 (1390,1393),
     * causal attention (1406-1429), output gate (1441-1444). */
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int i = 0; i < nrows; i++) {
        for (int h = 0; h < H; h++) {
            int t1 = rows[i];
            float* qrow = (float*)malloc(sizeof(float) * q_dim);
            float* scores = (float*)malloc(sizeof(float) * ((size_t)t1 + 1));
            for (int hh = 0; hh < H; hh++) {
                for (int d = 0; d < D; d++) {
                    size_t idx = (size_t)t1 * 2 * q_dim + (size_t)hh * 2 * D + d;
                    qrow[(size_t)hh * D + d] = q_gate_f32 ? q_gate_f32[idx] : bf16_to_f32(q_gate_bf16[idx]);
                }
            }
            per_head_rms_norm(qrow, H, D, q_norm);
            apply_partial_rope(qrow, H, D, cos_t, sin_t, rot, t1);
            float* o = out + (size_t)i * q_dim + (size_t)h * D;
            attend_one(qrow + (size_t)h * D, k_all, v_all, (int64_t)t1 + 1, kv_dim,
                       (h / groups) * D, D, scale, scores, o);
            for (int d = 0; d < D; d++) {
                size_t gidx = (size_t)t1 * 2 * q_dim + (size_t)h * 2 * D + D + d;
                float g = q_gate_f32 ? q_gate_f32[gidx] : bf16_to_f32(q_gate_bf16[gidx]);
                o[d] *= 1.0f / (1.0f + expf(-g));
            }
            free(qrow);
            free(scores);
        }
    }
    free(k_all);
    free(v_all);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Projections around the mixers: Q4 and F16 weight GEMV               */
/* ------------------------------------------------------------------ */

/* Q4 symmetric quantization of a [k][n] f32 matrix, groups of 32 along n
 * (src/convert.rs:437-467): scale = absmax / 7 stored as f16, values
 * round(x / scale) (half away from zero, with the f32 scale) clamped to
 * [-8, 7] and offset by 8, two per byte, the even column in the low nibble. */
void or_quantize_q4(const float* w, int k, int n, uint8_t* packed, uint16_t* scales) {
    const int gs = 32, groups = n / gs;
    for (int ki = 0; ki < k; ki++)
        for (int g = 0; g < groups; g++) {
            const float* grp = w + (size_t)ki * n + (size_t)g * gs;
            float absmax = 0.0f;
            for (int j = 0; j < gs; j++) absmax = fmaxf(absmax, fabsf(grp[j]));
            const float scale = absmax > 0.0f ? absmax / 7.0f : 0.0f;
            _Float16 sh = (_Float16)scale;
            memcpy(&scales[(size_t)ki * groups + g], &sh, 2);
            const float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
            uint8_t* dst = packed + (size_t)ki * (n / 2) + (size_t)g * (gs / 2);
            for (int j = 0; j < gs; j += 2) {
                int q0 = (int)roundf(grp[j] * inv), q1 = (int)roundf(grp[j + 1] * inv);
                q0 = (q0 < -8 ? -8 : q0 > 7 ? 7 : q0) + 8;
                q1 = (q1 < -8 ? -8 : q1 > 7 ? 7 : q1) + 8;
                dst[j / 2] = (uint8_t)(q0 | (q1 << 4));
            }
        }
}

static inline float f16_bits_to_f32(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

/* y[n] = x[k] . W[k][n] for Q4 W (src/gemv.rs:411-450, the scalar path):
 * rows with x == 0 and groups with scale * x == 0 are skipped; per group a
 * 16-entry table s * (q - 8) with s = scale * x; f32 sums in row order. */
void or_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales, int k, int n, float* y) {
    const int gs = 32, groups = n / gs;
    for (int j = 0; j < n; j++) y[j] = 0.0f;
    for (int ki = 0; ki < k; ki++) {
        const float val = x[ki];
        if (val == 0.0f) continue;
        for (int g = 0; g < groups; g++) {
            const float s = f16_bits_to_f32(scales[(size_t)ki * groups + g]) * val;
            if (s == 0.0f) continue;
            float lut[16];
            for (int i = 0; i < 16; i++) lut[i] = s * (float)(i - 8);
            const uint8_t* src = packed + (size_t)ki * (n / 2) + (size_t)g * (gs / 2);
            float* o = y + (size_t)g * gs;
            for (int jj = 0; jj < gs / 2; jj++) {
                o[2 * jj] += lut[src[jj] & 0x0F];
                o[2 * jj + 1] += lut[src[jj] >> 4];
            }
        }
    }
}

/* y[n] = x[k] . W[k][n] for F16 W (src/gemv.rs:361-368, the scalar path). */
void or_gemv_f16(const float* x, const uint16_t* w, int k, int n, float* y) {
    for (int j = 0; j < n; j++) y[j] = 0.0f;
    for (int ki = 0; ki < k; ki++) {
        const float val = x[ki];
        const uint16_t* row = w + (size_t)ki * n;
        for (int j = 0; j < n; j++) y[j] += val * f16_bits_to_f32(row[j]);
    }
}

/* ------------------------------------------------------------------ */
/* lm_head, logit penalties and sampling (the decode loop's tail)      */
/* ------------------------------------------------------------------ */

/* y[v] = x[hidden] . E[v][hidden] over the tied embedding rows, F16
 * (src/gemv.rs:664-676): f32 products added in column order per row. */
void or_lm_head_f16(const float* x, const uint16_t* e, int vocab, int hidden, float* y) {
    for (int v = 0; v < vocab; v++) {
        const uint16_t* row = e + (size_t)v * hidden;
        float sum = 0.0f;
        for (int j = 0; j < hidden; j++) sum += x[j] * f16_bits_to_f32(row[j]);
        y[v] = sum;
    }
}

/* The same for Q4 rows (src/gemv.rs:677-707): packed [vocab][hidden/2],
 * scales [vocab][hidden/32]; groups with scale 0 are skipped, per group a
 * table scale * (q - 8), dot += x[j] * table[q] in column order. */
void or_lm_head_q4(const float* x, const uint8_t* packed, const uint16_t* scales, int vocab, int hidden,
                   float* y) {
    const int gs = 32, groups = hidden / gs;
    for (int v = 0; v < vocab; v++) {
        float dot = 0.0f;
        for (int g = 0; g < groups; g++) {
            const float scale = f16_bits_to_f32(scales[(size_t)v * groups + g]);
            if (scale == 0.0f) continue;
            float lut[16];
            for (int i = 0; i < 16; i++) lut[i] = scale * (float)(i - 8);
            const uint8_t* src = packed + (size_t)v * (hidden / 2) + (size_t)g * (gs / 2);
            const float* xi = x + (size_t)g * gs;
            for (int jj = 0; jj < gs / 2; jj++) {
                dot += xi[2 * jj] * lut[src[jj] & 0x0F];
                dot += xi[2 * jj + 1] * lut[src[jj] >> 4];
            }
        }
        y[v] = dot;
    }
}

/* Repetition penalty (src/generate.rs:58-69): over the last min(len, 64)
 * generated tokens, each occurrence divides a positive logit by the penalty
 * or multiplies a non-positive one; nothing when penalty <= 1. */
void or_repetition_penalty(float* logits, int vocab, const int32_t* gen, int len, float penalty) {
    if (penalty <= 1.0f) return;
    const int window = len < 64 ? len : 64;
    for (int i = len - window; i < len; i++) {
        const int idx = gen[i];
        if (idx >= 0 && idx < vocab) {
            if (logits[idx] > 0.0f) logits[idx] /= penalty;
            else logits[idx] *= penalty;
        }
    }
}

/* Presence penalty (src/generate.rs:72-83): every token seen at least once
 * in the whole history loses `penalty` once; nothing when penalty <= 0 or the
 * history is empty. */
void or_presence_penalty(float* logits, int vocab, const int32_t* gen, int len, float penalty) {
    if (penalty <= 0.0f || len == 0) return;
    unsigned char* seen = (unsigned char*)calloc((size_t)vocab, 1);
    for (int i = 0; i < len; i++)
        if (gen[i] >= 0 && gen[i] < vocab) seen[gen[i]] = 1;
    for (int v = 0; v < vocab; v++)
        if (seen[v]) logits[v] -= penalty;
    free(seen);
}

typedef struct {
    int id;
    float val;
} or_cand;

static int cand_desc(const void* a, const void* b) {
    const or_cand* x = (const or_cand*)a;
    const or_cand* y = (const or_cand*)b;
    if (x->val > y->val) return -1;
    if (x->val < y->val) return 1;
    return x->id < y->id ? -1 : (x->id > y->id);  /* a stable sort keeps index order on ties */
}

/* sample_token_top_k (src/generate.rs:334-384) with the random draw r
 * (rng.next_f32()) given.  Returns the token; *margin (when not NULL) is
 * the smallest relative distance between a decision and its threshold
 * (the top-p cutoff, where moving it would change the candidates' mass by
 * more than 1e-5, and the draw against the running sums), so a test can
 * tell a boundary case from a mismatch.  Logits must not be NaN (the
 * reference's sort order is unspecified then). */
int or_sample_top_k(const float* logits, int vocab, float temperature, float top_p, int top_k, float r,
                    double* margin) {
    if (margin) *margin = 1.0;
    if (temperature <= 0.0f) {
        int best = 0;
        float bv = -INFINITY;
        for (int i = 0; i < vocab; i++)
            if (logits[i] > bv) {
                bv = logits[i];
                best = i;
            }
        return best;
    }
    const float inv_temp = 1.0f / temperature;
    float max_logit = -INFINITY;
    for (int i = 0; i < vocab; i++) max_logit = fmaxf(max_logit, logits[i]);
    or_cand* c = (or_cand*)malloc(sizeof(or_cand) * (size_t)vocab);
    for (int i = 0; i < vocab; i++) {
        c[i].id = i;
        c[i].val = logits[i];
    }
    qsort(c, (size_t)vocab, sizeof(or_cand), cand_desc);
    const int k = top_k > 0 ? (top_k < vocab ? top_k : vocab) : vocab;
    float* p = (float*)malloc(sizeof(float) * (size_t)k);
    float sum = 0.0f;
    for (int i = 0; i < k; i++) {
        p[i] = expf((c[i].val - max_logit) * inv_temp);
        sum += p[i];
    }
    int out;
    if (sum <= 0.0f) {
        out = c[0].id;
    } else {
        const float inv = 1.0f / sum;
        for (int i = 0; i < k; i++) p[i] *= inv;
        float cum = 0.0f;
        int cutoff = k;
        for (int i = 0; i < k; i++) {
            cum += p[i];
            /* a cut that flips here moves the candidate mass by ~(1 - cum):
             * a boundary only when that is more than rounding */
            if (margin && top_p != 0.0f && 1.0 - (double)cum > 1e-5) {
                const double d = fabs((double)cum - (double)top_p) / fabs((double)top_p);
                if (d < *margin) *margin = d;
            }
            if (cum >= top_p) {
                cutoff = i + 1;
                break;
            }
        }
        float total = 0.0f;
        for (int i = 0; i < cutoff; i++) total += p[i];
        if (total <= 0.0f) {
            out = c[0].id;
        } else {
            const float rv = r * total;
            float acc = 0.0f;
            out = c[0].id;
            for (int i = 0; i < cutoff; i++) {
                acc += p[i];
                if (margin && rv != 0.0f) {
                    const double d = fabs((double)acc - (double)rv) / (double)total;
                    if (d < *margin) *margin = d;
                }
                if (acc >= rv) {
                    out = c[i].id;
                    break;
                }
            }
        }
    }
    free(p);
    free(c);
    return out;
}

/* The reference's xorshift64 generator (src/generate.rs:41-55), for tests
 * that draw r the way the reference's decode loop does. */
float or_rng_next_f32(uint64_t* state) {
    uint64_t s = *state;
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    *state = s;
    return (float)(s >> 40) / 16777216.0f;
}
