// DeltaNet decode of T sequential tokens in one launch, the state on chip.
//
// The same per-token arithmetic as dn_decode.cu (conv1d(k=4) + SiLU, L2 norm
// of q and k with q * 1/sqrt(128), alpha/beta, then per state row
//     S1 = alpha*S;  p = S1.k;  d = beta*(v - p);  S2 = S1 + d k^T;  y = S2.q)
// applied to T tokens in order, which is the reference's per-token loop
// (src/gemv.rs:1129-1203 of prefill_deltanet_layer; T successive mixer
// regions of forward_deltanet_decode, src/gemv.rs:744-883, when the inputs
// are known ahead).  One CTA of 512 threads owns one (sequence, V head): its
// 64 KB state lives in registers for the whole call (4 lanes per 128-float
// row, 8 float4 each), so HBM sees one read and one write of S per call
// instead of per token.  The inputs of the next tokens stream into a ring of
// shared-memory slots by cp.async (kDepth tokens ahead); per token a CTA
// runs two barriers (three with the fused gate): inputs landed, then the
// conv/SiLU outputs and the norms' partial sums published.
#include "qm_internal.h"

namespace qm {
namespace {

constexpr int kSeqThreads = 512;
constexpr int kDepth = 8;             // tokens in flight per CTA
constexpr int kSlotF = 3 * kHd + kHd + 4;  // q, k, v raw; z raw; a, b (+pad), floats

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

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

template <bool GATE>
__global__ void __launch_bounds__(kSeqThreads, 1)
dn_decode_seq_kernel(const float* __restrict__ qkv, const float* __restrict__ a_in,
                     const float* __restrict__ b_in, const float* __restrict__ conv_w,
                     const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                     const float* __restrict__ norm_gamma, float* __restrict__ S,
                     float* __restrict__ conv, int64_t conv_pos, int T, float* __restrict__ y,
                     const float* __restrict__ z, float* __restrict__ out, int vh_lo, int nvh) {
    const int lh = blockIdx.x;  // head within the state's range
    const int vh = vh_lo + lh;  // model V head
    const int qk = vh >> 1;     // GVA: V head vh reads QK head vh/2 (gemv.rs:803-809)
    const int b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lane4 = lane & 3;
    const int row = warp * 8 + (lane >> 2);  // state row (v dim) of this lane

    __shared__ __align__(16) float s_in[kDepth][kSlotF];
    __shared__ __align__(16) float s_act[3 * kHd];  // q, k, v after conv + SiLU
    __shared__ float s_red[8];                       // sum of squares: q warps 0-3, k warps 4-7
    __shared__ float s_ab[2];
    __shared__ float s_ysq[16];

    // ---- the state rows, once (4 lanes per row, float4 chunk 4j + lane4) ----
    float* Sh = S + ((size_t)(b * nvh + lh) * kHd + row) * kHd;
    float4 sr[8];
#pragma unroll
    for (int j = 0; j < 8; j++) sr[j] = reinterpret_cast<const float4*>(Sh)[4 * j + lane4];

    // ---- input streaming: token t -> slot t % kDepth ----
    const size_t tok0 = (size_t)b * T;
    auto issue = [&](int t) {
        if (t < T) {
            float* d = s_in[t % kDepth];
            const float* x = qkv + (tok0 + t) * kQKVDim;
            if (tid < 96) {  // q, k, v: 3 x 32 chunks of 16 bytes
                const int part = tid >> 5, c = tid & 31;
                const float* src = part == 0 ? x + qk * kHd : part == 1 ? x + kQDim + qk * kHd
                                                                        : x + 2 * kQDim + vh * kHd;
                cp_async16(d + part * kHd + 4 * c, src + 4 * c);
            } else if (GATE && tid < 128) {
                const int c = tid - 96;
                cp_async16(d + 3 * kHd + 4 * c, z + (tok0 + t) * kVDim + (size_t)vh * kHd + 4 * c);
            } else if (tid == 128) {
                cp_async4(d + 4 * kHd, a_in + (tok0 + t) * kNumV + vh);
            } else if (tid == 129) {
                cp_async4(d + 4 * kHd + 1, b_in + (tok0 + t) * kNumV + vh);
            }
        }
        cp_async_commit();  // one group per token, empty past the end
    };
#pragma unroll 1
    for (int t = 0; t < kDepth - 1; t++) issue(t);

    // ---- conv history and taps of this thread's channel (threads < 384) ----
    // channel order in a slot: q [0,128), k [128,256), v [256,384)
    int ch = -1;
    if (tid < kHd) ch = qk * kHd + tid;
    else if (tid < 2 * kHd) ch = kQDim + qk * kHd + (tid - kHd);
    else if (tid < 3 * kHd) ch = 2 * kQDim + vh * kHd + (tid - 2 * kHd);
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    float h1 = 0.f, h2 = 0.f, h3 = 0.f;  // inputs of tokens t-1, t-2, t-3
    float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
    if (ch >= 0) {
        w = reinterpret_cast<const float4*>(conv_w)[ch];
        h3 = ring[((conv_pos + 1) & 3) * kQKVDim + ch];  // slot of token conv_pos - 3
        h2 = ring[((conv_pos + 2) & 3) * kQKVDim + ch];
        h1 = ring[((conv_pos + 3) & 3) * kQKVDim + ch];
    }
    const float a_exp = __expf(a_log[vh]);
    const float dtb = dt_bias[vh];
    const float gam = GATE ? norm_gamma[row] : 0.f;
    float* yb = y ? y + (tok0 * nvh + lh) * kHd + row : nullptr;
    float* ob = GATE ? out + (tok0 * nvh + lh) * kHd + row : nullptr;
    const size_t tstride = (size_t)nvh * kHd;

#pragma unroll 1
    for (int t = 0; t < T; t++) {
        issue(t + kDepth - 1);  // into the slot of token t-1, which nobody reads any more
        cp_async_wait<kDepth - 1>();
        __syncthreads();  // token t's inputs visible to every thread
        const float* d = s_in[t % kDepth];

        // conv1d(k=4) + SiLU (gemv.rs:744-772); q/k partial sums of squares
        if (ch >= 0) {
            const float x0 = d[tid];
            float c = h3 * w.x;
            c += h2 * w.y;
            c += h1 * w.z;
            c += x0 * w.w;
            h3 = h2;
            h2 = h1;
            h1 = x0;
            const float act = silu_f(c);
            s_act[tid] = act;
            if (tid < 2 * kHd) {
                float sq = act * act;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) s_red[warp] = sq;
            }
        } else if (tid == kSeqThreads - 1) {
            // alpha/beta (gemv.rs:791-800)
            const float sp = softplus_f(d[4 * kHd] + dtb);
            s_ab[0] = __expf(-a_exp * sp);
            s_ab[1] = 1.0f / (1.0f + __expf(-d[4 * kHd + 1]));
        }
        const float zr = GATE ? d[3 * kHd + row] : 0.f;
        __syncthreads();  // activations, partial sums and gates published

        // l2_normalize (gemv.rs:641-649), q * 1/sqrt(128) (784)
        const float nq = sqrtf(s_red[0] + s_red[1] + s_red[2] + s_red[3]);
        const float nk = sqrtf(s_red[4] + s_red[5] + s_red[6] + s_red[7]);
        const float iq = nq > 1e-12f ? 1.0f / nq : 1.0f;
        const float ik = nk > 1e-12f ? 1.0f / nk : 1.0f;
        const float alpha = s_ab[0], beta = s_ab[1];
        const float vr = s_act[2 * kHd + row];
        const float4* q4 = reinterpret_cast<const float4*>(s_act);
        const float4* k4 = reinterpret_cast<const float4*>(s_act + kHd);

        float p0 = 0.f, p1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 kk = k4[4 * j + lane4];
            float4& s = sr[j];
            s.x *= alpha; s.y *= alpha; s.z *= alpha; s.w *= alpha;
            p0 = fmaf(s.x, kk.x * ik, p0);
            p1 = fmaf(s.y, kk.y * ik, p1);
            p0 = fmaf(s.z, kk.z * ik, p0);
            p1 = fmaf(s.w, kk.w * ik, p1);
        }
        float pk = p0 + p1;
        pk += __shfl_xor_sync(0xffffffffu, pk, 1);
        pk += __shfl_xor_sync(0xffffffffu, pk, 2);
        const float delta = beta * (vr - pk);
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 kk = k4[4 * j + lane4];
            const float4 qq = q4[4 * j + lane4];
            float4& s = sr[j];
            s.x = fmaf(delta, kk.x * ik, s.x);
            s.y = fmaf(delta, kk.y * ik, s.y);
            s.z = fmaf(delta, kk.z * ik, s.z);
            s.w = fmaf(delta, kk.w * ik, s.w);
            y0 = fmaf(s.x, (qq.x * iq) * 0.08838834764831845f, y0);
            y1 = fmaf(s.y, (qq.y * iq) * 0.08838834764831845f, y1);
            y0 = fmaf(s.z, (qq.z * iq) * 0.08838834764831845f, y0);
            y1 = fmaf(s.w, (qq.w * iq) * 0.08838834764831845f, y1);
        }
        float yr = y0 + y1;
        yr += __shfl_xor_sync(0xffffffffu, yr, 1);
        yr += __shfl_xor_sync(0xffffffffu, yr, 2);
        if (lane4 == 0 && yb) yb[(size_t)t * tstride] = yr;

        if constexpr (GATE) {
            // per-head RMSNorm (plain gamma) * SiLU(z) (gemv.rs:864-883)
            float sq = lane4 == 0 ? yr * yr : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (lane == 0) s_ysq[warp] = sq;
            __syncthreads();
            float tot = 0.f;
#pragma unroll
            for (int i = 0; i < 16; i++) tot += s_ysq[i];
            const float inv_rms = 1.0f / sqrtf(tot * (1.0f / kHd) + 1e-6f);
            if (lane4 == 0) ob[(size_t)t * tstride] = yr * inv_rms * gam * silu_f(zr);
        }
    }
    cp_async_wait<0>();  // nothing may land after the CTA exits

    // ---- the state back, and the conv history of the last three tokens ----
#pragma unroll
    for (int j = 0; j < 8; j++) reinterpret_cast<float4*>(Sh)[4 * j + lane4] = sr[j];
    // q/k channels are shared by V heads 2qk and 2qk+1: the even one writes them
    if (ch >= 0 && (tid >= 2 * kHd || (vh & 1) == 0)) {
        const int64_t e = conv_pos + T;  // next token; its history is e-3 .. e-1
        ring[((e - 1) & 3) * kQKVDim + ch] = h1;
        ring[((e - 2) & 3) * kQKVDim + ch] = h2;
        ring[((e - 3) & 3) * kQKVDim + ch] = h3;
    }
}

}  // namespace

cudaError_t launch_dn_decode_seq(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                                 const float* qkv, const float* a, const float* b, float* y,
                                 const float* z, float* out) {
    dim3 grid(st->nvh, st->batch);
    TimedLaunch tl(ctx, "dn_decode_seq");
    if (z)
        dn_decode_seq_kernel<true><<<grid, kSeqThreads, 0, ctx->stream>>>(
            qkv, a, b, p->conv_w, p->a_log, p->dt_bias, p->norm_gamma, st->s, st->conv, st->conv_pos, T,
            y, z, out, st->vh_lo, st->nvh);
    else
        dn_decode_seq_kernel<false><<<grid, kSeqThreads, 0, ctx->stream>>>(
            qkv, a, b, p->conv_w, p->a_log, p->dt_bias, nullptr, st->s, st->conv, st->conv_pos, T, y,
            nullptr, nullptr, st->vh_lo, st->nvh);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) ctx->launches += 1;
    return e;
}

}  // namespace qm
