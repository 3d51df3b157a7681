// DeltaNet decode of T sequential tokens in one launch, the state on chip.
//
// The per-token arithmetic of dn_decode.cu (conv1d(k=4) + SiLU, L2 norm of q
// and k with q * 1/sqrt(128), alpha/beta, then per state row
//     S1 = alpha*S;  p = S1.k;  d = beta*(v - p);  S2 = S1 + d k^T;  y = S2.q)
// — with the two norm factors applied to the row sums instead of the
// vectors, 4 operations per state element and token instead of 8 — applied
// to T tokens in order, which is the reference's per-token loop
// (src/gemv.rs:1129-1203 of prefill_deltanet_layer; T successive mixer
// regions of forward_deltanet_decode, src/gemv.rs:744-883, when the inputs
// are known ahead).  Four CTAs of 512 threads own one (sequence, V head),
// 32 state rows each, held in registers for the whole call (16 lanes per
// 128-float row, two float4 each), so HBM sees one read and one write of S
// per call instead of per token.  Only the state update is sequential:
// conv, SiLU, the norms and the gates of 32 tokens are computed together
// (their inputs stream in by cp.async while the previous 32 tokens run), and
// each row then walks those tokens with no barrier.  The optional RMSNorm *
// SiLU(z) gate runs afterwards as one elementwise launch over all tokens.
#include "qm_internal.h"

namespace qm {
namespace {

constexpr int kSplit = 4;                    // CTAs per V head
constexpr int kRows = kHd / kSplit;          // state rows per CTA
constexpr int kLanes = 16;                   // lanes per row (two float4 each)
constexpr int kSeqThreads = kLanes * kRows;  // 512
constexpr int kChunk = 32;                   // tokens prepared together
constexpr int kActF = 2 * kHd + kRows;       // q, k, this block's v: 288 floats per token
constexpr int kRawF = kActF + 4;             // + a, b (+ pad): 292 floats = 1168 bytes
constexpr int kRawBytes = 2 * kChunk * kRawF * 4;  // double-buffered raw inputs
constexpr int kActBytes = kChunk * kActF * 4;
constexpr int kScBytes = kChunk * 4 * 4;           // per token: k scale, q scale, alpha, beta
constexpr int kSeqSmem = kRawBytes + kActBytes + kScBytes;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }
// SiLU with the approximate division (2 ulp)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(__expf(x)); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One CTA per (sequence, V head, quarter of the head's 128 state rows): 16
// lanes per row, 32 rows, 512 threads.  Every CTA of a head computes the
// head's q and k itself, so the CTAs never communicate.  Per chunk of 32
// tokens:
//   1. the chunk's raw inputs are in shared memory (loaded by cp.async while
//      the previous chunk ran);
//   2. conv1d + SiLU for the 288 channels (one channel per thread, the
//      chunk's tokens independent of each other) and the gates alpha, beta;
//   3. the 64 L2 norms of the chunk's q and k (warp reductions);
//   4. the recurrence: each row walks the chunk's tokens with no barrier —
//      only the state update is sequential.  The reduction of y for token t
//      runs in the same shuffle steps as the state-row sum of token t + 1.
__global__ void __launch_bounds__(kSeqThreads)
dn_decode_seq_kernel(const float* __restrict__ qkv, const float* __restrict__ a_in,
                     const float* __restrict__ b_in, const float* __restrict__ conv_w,
                     const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                     float* __restrict__ S, float* __restrict__ conv, int64_t conv_pos, int T,
                     float* __restrict__ y, int vh_lo, int nvh) {
    extern __shared__ __align__(16) float smem[];
    float* s_raw = smem;                                  // [2][kChunk][kRawF]
    float* s_act = smem + 2 * kChunk * kRawF;             // [kChunk][kActF]
    float4* s_sc = reinterpret_cast<float4*>(s_act + kChunk * kActF);  // [kChunk]

    const int lh = blockIdx.x / kSplit;  // head within the state's range
    const int part = blockIdx.x % kSplit;
    const int vh = vh_lo + lh;           // model V head
    const int qk = vh >> 1;              // GVA: V head vh reads QK head vh/2 (gemv.rs:803-809)
    const int b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int l16 = tid & (kLanes - 1);
    const int lrow = tid / kLanes;        // row within this CTA's block
    const int row = part * kRows + lrow;  // state row (v dim)
    const int nchunks = (T + kChunk - 1) / kChunk;

    // ---- the state rows, once (float4 chunks l16 and l16 + 16 of the row) ----
    float* Sh = S + ((size_t)(b * nvh + lh) * kHd + row) * kHd;
    float4 sr[2];
#pragma unroll
    for (int j = 0; j < 2; j++) sr[j] = reinterpret_cast<const float4*>(Sh)[kLanes * j + l16];

    // ---- raw inputs of chunk c into buffer c & 1 ----
    const size_t tok0 = (size_t)b * T;
    auto issue = [&](int c) {
        if (c < nchunks) {
            const int t0 = c * kChunk, nt = min(kChunk, T - t0);
            float* d = s_raw + (c & 1) * kChunk * kRawF;
            for (int i = tid; i < nt * (kActF / 4); i += kSeqThreads) {
                const int t = i / (kActF / 4), j = i % (kActF / 4);  // 72 chunks of 16 bytes a token
                const float* x = qkv + (tok0 + t0 + t) * kQKVDim;
                const float* src = j < 32 ? x + qk * kHd + 4 * j
                                 : j < 64 ? x + kQDim + qk * kHd + 4 * (j - 32)
                                          : x + 2 * kQDim + vh * kHd + part * kRows + 4 * (j - 64);
                cp_async16(d + t * kRawF + 4 * j, src);
            }
            if (tid < 2 * nt) {
                const int t = tid >> 1;
                const float* src = ((tid & 1) ? b_in : a_in) + (tok0 + t0 + t) * kNumV + vh;
                cp_async4(d + t * kRawF + kActF + (tid & 1), src);
            }
        }
        cp_async_commit();  // one group per chunk, empty past the end
    };
    issue(0);

    // ---- conv history and taps: thread tid < 288 owns channel tid of a
    // token: q [0,128), k [128,256), this block's v [256,288) ----
    int ch = -1;
    if (tid < kHd) ch = qk * kHd + tid;
    else if (tid < 2 * kHd) ch = kQDim + qk * kHd + (tid - kHd);
    else if (tid < kActF) ch = 2 * kQDim + vh * kHd + part * kRows + (tid - 2 * kHd);
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    float h1 = 0.f, h2 = 0.f, h3 = 0.f;  // raw inputs of the last three tokens
    float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
    if (ch >= 0) {
        w = reinterpret_cast<const float4*>(conv_w)[ch];
        h3 = ring[((conv_pos + 1) & 3) * kQKVDim + ch];  // slot of token conv_pos - 3
        h2 = ring[((conv_pos + 2) & 3) * kQKVDim + ch];
        h1 = ring[((conv_pos + 3) & 3) * kQKVDim + ch];
    }
    const float a_exp = __expf(a_log[vh]);
    const float dtb = dt_bias[vh];
    float* yb = y + (tok0 * nvh + lh) * kHd + row;
    const size_t tstride = (size_t)nvh * kHd;
    const float4* act4 = reinterpret_cast<const float4*>(s_act);

    // y of the previous token: partial sum still to reduce, and its scale
    float ypend = 0.f, ypend_sc = 0.f;
    int ypend_t = -1;

#pragma unroll 1
    for (int c = 0; c < nchunks; c++) {
        const int t0 = c * kChunk, nt = min(kChunk, T - t0);
        issue(c + 1);  // into the buffer chunk c-1 used (its readers passed the barrier below)
        cp_async_wait<1>();
        __syncthreads();  // chunk c's raw inputs visible; chunk c-1's rows are done with s_act
        const float* d = s_raw + (c & 1) * kChunk * kRawF;

        // ---- 2. conv1d(k=4) + SiLU (gemv.rs:744-772), gates (gemv.rs:791-800) ----
        if (ch >= 0) {
#pragma unroll 8
            for (int t = 0; t < nt; t++) {
                const float x0 = d[t * kRawF + tid];
                float cv = h3 * w.x;
                cv += h2 * w.y;
                cv += h1 * w.z;
                cv += x0 * w.w;
                h3 = h2;
                h2 = h1;
                h1 = x0;
                s_act[t * kActF + tid] = silu_fast(cv);
            }
        } else if (tid < kActF + kChunk) {
            const int t = tid - kActF;
            if (t < nt) {
                const float sp = softplus_f(d[t * kRawF + kActF] + dtb);
                s_sc[t].z = __expf(-a_exp * sp);
                s_sc[t].w = 1.0f / (1.0f + __expf(-d[t * kRawF + kActF + 1]));
            }
        }
        __syncthreads();

        // ---- 3. l2_normalize (gemv.rs:641-649) of q and k, q * 1/sqrt(128) (784):
        // warp w reduces (token, q|k) pairs w, w + 16, w + 32, w + 48 ----
        {
            float sq[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int idx = warp + 16 * u, t = idx >> 1, which = idx & 1;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < nt) v = act4[t * (kActF / 4) + which * 32 + lane];
                sq[u] = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < 4; u++) sq[u] += __shfl_xor_sync(0xffffffffu, sq[u], o);
            if (lane < 4) {
                const int idx = warp + 16 * lane, t = idx >> 1, which = idx & 1;
                const float ssq = lane == 0 ? sq[0] : lane == 1 ? sq[1] : lane == 2 ? sq[2] : sq[3];
                if (t < nt) {
                    const float n = sqrtf(ssq);
                    const float inv = n > 1e-12f ? 1.0f / n : 1.0f;
                    if (which) s_sc[t].x = inv;                          // k
                    else s_sc[t].y = inv * 0.08838834764831845f;         // q, scaled
                }
            }
        }
        __syncthreads();

        // ---- 4. the recurrence over the chunk, norms folded into the row sums:
        //   p = ik (S1 . k),  S2 = alpha S + (beta (v - alpha ik (S . k)) ik) k,
        //   y = iq (S2 . q) ----
#pragma unroll 2
        for (int t = 0; t < nt; t++) {
            const float4 sc = s_sc[t];  // ik, iq, alpha, beta
            const float4 k0 = act4[t * (kActF / 4) + 32 + l16], k1 = act4[t * (kActF / 4) + 48 + l16];
            const float4 q0 = act4[t * (kActF / 4) + l16], q1 = act4[t * (kActF / 4) + 16 + l16];
            const float vr = s_act[t * kActF + 2 * kHd + lrow];
            float p0 = sr[0].x * k0.x, p1 = sr[0].y * k0.y, p2 = sr[0].z * k0.z, p3 = sr[0].w * k0.w;
            p0 = fmaf(sr[1].x, k1.x, p0);
            p1 = fmaf(sr[1].y, k1.y, p1);
            p2 = fmaf(sr[1].z, k1.z, p2);
            p3 = fmaf(sr[1].w, k1.w, p3);
            float pk = (p0 + p1) + (p2 + p3);
            // the row sum of this token and the y sum of the previous one, together
#pragma unroll
            for (int o = 1; o < kLanes; o <<= 1) {
                pk += __shfl_xor_sync(0xffffffffu, pk, o);
                ypend += __shfl_xor_sync(0xffffffffu, ypend, o);
            }
            if (l16 == 0 && ypend_t >= 0) yb[(size_t)ypend_t * tstride] = ypend * ypend_sc;
            const float alpha = sc.z;
            const float dk = sc.w * (vr - alpha * sc.x * pk) * sc.x;  // delta, times the k scale
            sr[0].x = fmaf(dk, k0.x, alpha * sr[0].x);
            sr[0].y = fmaf(dk, k0.y, alpha * sr[0].y);
            sr[0].z = fmaf(dk, k0.z, alpha * sr[0].z);
            sr[0].w = fmaf(dk, k0.w, alpha * sr[0].w);
            sr[1].x = fmaf(dk, k1.x, alpha * sr[1].x);
            sr[1].y = fmaf(dk, k1.y, alpha * sr[1].y);
            sr[1].z = fmaf(dk, k1.z, alpha * sr[1].z);
            sr[1].w = fmaf(dk, k1.w, alpha * sr[1].w);
            float y0 = sr[0].x * q0.x, y1 = sr[0].y * q0.y, y2 = sr[0].z * q0.z, y3 = sr[0].w * q0.w;
            y0 = fmaf(sr[1].x, q1.x, y0);
            y1 = fmaf(sr[1].y, q1.y, y1);
            y2 = fmaf(sr[1].z, q1.z, y2);
            y3 = fmaf(sr[1].w, q1.w, y3);
            ypend = (y0 + y1) + (y2 + y3);
            ypend_sc = sc.y;
            ypend_t = t0 + t;
        }
    }
    // the last token's y
#pragma unroll
    for (int o = 1; o < kLanes; o <<= 1) ypend += __shfl_xor_sync(0xffffffffu, ypend, o);
    if (l16 == 0 && ypend_t >= 0) yb[(size_t)ypend_t * tstride] = ypend * ypend_sc;
    cp_async_wait<0>();  // nothing may land after the CTA exits

    // ---- the state back, and the conv history of the last three tokens ----
#pragma unroll
    for (int j = 0; j < 2; j++) reinterpret_cast<float4*>(Sh)[kLanes * j + l16] = sr[j];
    const int64_t e = conv_pos + T;  // next token; its history is e-3 .. e-1
    const int w1 = (int)((e - 1) & 3), w2 = (int)((e - 2) & 3), w3 = (int)((e - 3) & 3);
    // q/k channels are shared by V heads 2qk and 2qk+1 and by the head's
    // quarters: the first quarter of the even head writes them
    if (ch >= 0 && (tid >= 2 * kHd || (part == 0 && (vh & 1) == 0))) {
        ring[w1 * kQKVDim + ch] = h1;
        ring[w2 * kQKVDim + ch] = h2;
        ring[w3 * kQKVDim + ch] = h3;
    }
}

// per-head RMSNorm (plain gamma) * SiLU(z) of y [B*T, nvh, 128] (gemv.rs:864-883):
// one warp per (token, head); may run in place (out == y)
__global__ void dn_seq_gate_kernel(const float* y, const float* __restrict__ z,
                                   const float* __restrict__ gamma, float* out, size_t rows, int vh_lo,
                                   int nvh) {
    const size_t wid = (size_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wid >= rows) return;
    const size_t tok = wid / nvh;
    const int vh = vh_lo + (int)(wid % nvh);
    const float4 v = reinterpret_cast<const float4*>(y + wid * kHd)[lane];
    float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / kHd) + 1e-6f);
    const float4 zz = reinterpret_cast<const float4*>(z + tok * kVDim + (size_t)vh * kHd)[lane];
    const float4 gg = reinterpret_cast<const float4*>(gamma)[lane];
    float4 o;
    o.x = v.x * inv * gg.x * silu_f(zz.x);
    o.y = v.y * inv * gg.y * silu_f(zz.y);
    o.z = v.z * inv * gg.z * silu_f(zz.z);
    o.w = v.w * inv * gg.w * silu_f(zz.w);
    reinterpret_cast<float4*>(out + wid * kHd)[lane] = o;
}

}  // namespace

cudaError_t launch_dn_decode_seq(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                                 const float* qkv, const float* a, const float* b, float* y,
                                 const float* z, float* out) {
    float* yw = y ? y : out;  // raw y goes to out first when only the gated output is wanted
    {
        static std::atomic<uint64_t> attr_set{0};
        const cudaError_t ea = set_smem_once(attr_set, ctx->device, dn_decode_seq_kernel, kSeqSmem);
        if (ea != cudaSuccess) return ea;
        dim3 grid(st->nvh * kSplit, st->batch);
        TimedLaunch tl(ctx, "dn_decode_seq");
        dn_decode_seq_kernel<<<grid, kSeqThreads, kSeqSmem, ctx->stream>>>(
            qkv, a, b, p->conv_w, p->a_log, p->dt_bias, st->s, st->conv, st->conv_pos, T, yw, st->vh_lo,
            st->nvh);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    if (z) {
        const size_t rows = (size_t)st->batch * T * st->nvh;
        dn_seq_gate_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, ctx->stream>>>(yw, z, p->norm_gamma, out,
                                                                                rows, st->vh_lo, st->nvh);
        e = cudaGetLastError();
        if (e == cudaSuccess) ctx->launches += 1;
    }
    return e;
}

}  // namespace qm
