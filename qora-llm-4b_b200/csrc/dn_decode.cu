// DeltaNet decode: one token for B sequences, one fused pass over the state.
//
// Replaces src/gemv.rs:744-883 (CPU) and src/gpu_inference.rs:149-227 (wgpu).
// The reference makes four passes over each 64 KB head state (decay,
// retrieve, delta update, output: simd.rs:304-361).  Here every state row is
// loaded once into registers, updated with the same operation sequence
//     S1 = alpha*S;  p = S1.k;  d = beta*(v - p);  S2 = S1 + d k^T;  y = S2.q
// and stored once, so HBM traffic is one read + one write of S.
//
// Thread layout: 256 threads; 8 lanes own one 128-float row (4 float4 each,
// interleaved so one warp instruction reads 4 full 128-byte row segments);
// a warp covers 4 rows per pass; row dot products reduce over the 8 lanes
// with 3 xor-shuffles.  A CTA owns ROWS = 128/SPLIT rows of one (seq, head).
// SPLIT > 1 spreads small batches over more SMs; the fused gate epilogue
// then needs the head's sum of squares from all SPLIT CTAs, which a
// thread-block cluster exchanges through distributed shared memory.
#include <cooperative_groups.h>

#include "qm_internal.h"

namespace cg = cooperative_groups;

namespace qm {
namespace {

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float softplus_f(float x) {
    // src/gemv.rs:637-639
    return x > 20.0f ? x : log1pf(__expf(x));
}

template <int SPLIT, bool FUSED>
__global__ void __launch_bounds__(256, 2)
dn_decode_kernel(const float* __restrict__ qkv, const float* __restrict__ a_in,
                 const float* __restrict__ b_in, const float* __restrict__ conv_w,
                 const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                 const float* __restrict__ norm_gamma, float* __restrict__ S,
                 float* __restrict__ conv, int slot_w, float* __restrict__ y,
                 const float* __restrict__ z, float* __restrict__ out, int vh_lo, int nvh, int b0) {
    constexpr int ROWS = kHd / SPLIT;
    constexpr int PASSES = ROWS / 32;
    static_assert(PASSES >= 1, "ROWS must be a multiple of 32");

    const int lh = blockIdx.x / SPLIT;  // head within the state's range
    const int vh = vh_lo + lh;          // model V head (inputs, params, conv channels)
    const int part = blockIdx.x % SPLIT;
    const int b = b0 + blockIdx.y;  // sequences [b0, b0 + gridDim.y) of the batch
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int lane8 = lane & 7;
    const int rsub = lane >> 3;

    __shared__ float s_qk[2][kHd];  // q (scaled), k after conv/SiLU/L2
    __shared__ float s_v[kHd];
    __shared__ float s_red[2][4];
    __shared__ float s_ab[2];
    __shared__ float s_y[ROWS];
    __shared__ float s_wsq[8];
    __shared__ float s_sq;

    // ---- 1. issue the state loads first (they overlap the prologue) ----
    float* Sh = S + ((size_t)(b * nvh + lh) * kHd + part * ROWS) * kHd;
    float4 sr[PASSES][4];
#pragma unroll
    for (int p = 0; p < PASSES; p++) {
        const int r = p * 32 + warp * 4 + rsub;
        const float4* row = reinterpret_cast<const float4*>(Sh + (size_t)r * kHd);
#pragma unroll
        for (int j = 0; j < 4; j++) sr[p][j] = row[j * 8 + lane8];
    }

    // ---- 2. prologue: conv1d(k=4) + SiLU + L2 norm (gemv.rs:744-785) ----
    const int qk = vh >> 1;  // GVA: V head vh reads QK head vh/2 (gemv.rs:803-809)
    const float* x = qkv + (size_t)b * kQKVDim;
    float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
    const int s0 = (slot_w + 1) & 3, s1 = (slot_w + 2) & 3, s2 = (slot_w + 3) & 3;
    const bool writer = (part == 0);
    float qv = 0.f, kv = 0.f;
    if (tid < kHd) {
        const int chq = qk * kHd + tid;
        const int chk = kQDim + qk * kHd + tid;
        const float4 wq = reinterpret_cast<const float4*>(conv_w)[chq];
        const float4 wk = reinterpret_cast<const float4*>(conv_w)[chk];
        const float xq = x[chq], xk = x[chk];
        float cq = ring[s0 * kQKVDim + chq] * wq.x;
        cq += ring[s1 * kQKVDim + chq] * wq.y;
        cq += ring[s2 * kQKVDim + chq] * wq.z;
        cq += xq * wq.w;
        float ck = ring[s0 * kQKVDim + chk] * wk.x;
        ck += ring[s1 * kQKVDim + chk] * wk.y;
        ck += ring[s2 * kQKVDim + chk] * wk.z;
        ck += xk * wk.w;
        qv = silu_f(cq);
        kv = silu_f(ck);
        if (writer && (vh & 1) == 0) {  // one CTA per QK head advances its history
            ring[slot_w * kQKVDim + chq] = xq;
            ring[slot_w * kQKVDim + chk] = xk;
        }
    } else {
        const int c = tid - kHd;
        const int chv = 2 * kQDim + vh * kHd + c;
        const float4 wv = reinterpret_cast<const float4*>(conv_w)[chv];
        const float xv = x[chv];
        float cv = ring[s0 * kQKVDim + chv] * wv.x;
        cv += ring[s1 * kQKVDim + chv] * wv.y;
        cv += ring[s2 * kQKVDim + chv] * wv.z;
        cv += xv * wv.w;
        s_v[c] = silu_f(cv);
        if (writer) ring[slot_w * kQKVDim + chv] = xv;
    }
    if (tid < kHd) {
        float sq = qv * qv, sk = kv * kv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        if (lane == 0) {
            s_red[0][warp] = sq;
            s_red[1][warp] = sk;
        }
    }
    if (tid == 255) {
        // alpha/beta (gemv.rs:791-800)
        const float a_exp = __expf(a_log[vh]);
        const float sp = softplus_f(a_in[b * kNumV + vh] + dt_bias[vh]);
        s_ab[0] = __expf(-a_exp * sp);
        s_ab[1] = 1.0f / (1.0f + __expf(-b_in[b * kNumV + vh]));
    }
    __syncthreads();
    if (tid < kHd) {
        // l2_normalize (gemv.rs:641-649) then q *= 1/sqrt(128) (784)
        const float nq = sqrtf(s_red[0][0] + s_red[0][1] + s_red[0][2] + s_red[0][3]);
        const float nk = sqrtf(s_red[1][0] + s_red[1][1] + s_red[1][2] + s_red[1][3]);
        if (nq > 1e-12f) qv *= 1.0f / nq;
        if (nk > 1e-12f) kv *= 1.0f / nk;
        s_qk[0][tid] = qv * 0.08838834764831845f;  // 1/sqrt(128) in f32
        s_qk[1][tid] = kv;
    }
    __syncthreads();

    // ---- 3. fused state update (simd.rs:304-361 in one pass) ----
    const float alpha = s_ab[0], beta = s_ab[1];
    float4 kr[4], qr[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        kr[j] = reinterpret_cast<const float4*>(s_qk[1])[j * 8 + lane8];
        qr[j] = reinterpret_cast<const float4*>(s_qk[0])[j * 8 + lane8];
    }
    float* yb = y ? y + ((size_t)b * nvh + lh) * kHd + part * ROWS : nullptr;
    float sq_part = 0.f;
#pragma unroll
    for (int p = 0; p < PASSES; p++) {
        const int r = p * 32 + warp * 4 + rsub;
        const float vr = s_v[part * ROWS + r];
        float pk0 = 0.f, pk1 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4& s = sr[p][j];
            s.x *= alpha; s.y *= alpha; s.z *= alpha; s.w *= alpha;
            pk0 = fmaf(s.x, kr[j].x, pk0);
            pk1 = fmaf(s.y, kr[j].y, pk1);
            pk0 = fmaf(s.z, kr[j].z, pk0);
            pk1 = fmaf(s.w, kr[j].w, pk1);
        }
        float pk = pk0 + pk1;
        pk += __shfl_xor_sync(0xffffffffu, pk, 1);
        pk += __shfl_xor_sync(0xffffffffu, pk, 2);
        pk += __shfl_xor_sync(0xffffffffu, pk, 4);
        const float delta = beta * (vr - pk);
        float py0 = 0.f, py1 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4& s = sr[p][j];
            s.x = fmaf(delta, kr[j].x, s.x);
            s.y = fmaf(delta, kr[j].y, s.y);
            s.z = fmaf(delta, kr[j].z, s.z);
            s.w = fmaf(delta, kr[j].w, s.w);
            py0 = fmaf(s.x, qr[j].x, py0);
            py1 = fmaf(s.y, qr[j].y, py1);
            py0 = fmaf(s.z, qr[j].z, py0);
            py1 = fmaf(s.w, qr[j].w, py1);
        }
        float yr = py0 + py1;
        yr += __shfl_xor_sync(0xffffffffu, yr, 1);
        yr += __shfl_xor_sync(0xffffffffu, yr, 2);
        yr += __shfl_xor_sync(0xffffffffu, yr, 4);
        float4* row = reinterpret_cast<float4*>(Sh + (size_t)r * kHd);
#pragma unroll
        for (int j = 0; j < 4; j++) row[j * 8 + lane8] = sr[p][j];
        if (lane8 == 0) {
            if (yb) yb[r] = yr;
            if (FUSED) {
                s_y[r] = yr;
                sq_part += yr * yr;
            }
        }
    }

    // ---- 4. optional epilogue: RMSNorm(y)*gamma*SiLU(z) (gemv.rs:864-883) ----
    if constexpr (FUSED) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq_part += __shfl_xor_sync(0xffffffffu, sq_part, o);
        if (lane == 0) s_wsq[warp] = sq_part;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < 8; w++) t += s_wsq[w];
            s_sq = t;
        }
        __syncthreads();
        float total;
        if constexpr (SPLIT > 1) {
            cg::cluster_group cl = cg::this_cluster();
            cl.sync();
            total = 0.f;
#pragma unroll
            for (int r = 0; r < SPLIT; r++) total += *cl.map_shared_rank(&s_sq, r);
            cl.sync();
        } else {
            total = s_sq;
        }
        const float inv_rms = 1.0f / sqrtf(total * (1.0f / kHd) + 1e-6f);
        if (tid < ROWS) {
            const int c = part * ROWS + tid;
            const float yn = s_y[tid] * inv_rms * norm_gamma[c];
            out[((size_t)b * nvh + lh) * kHd + c] = yn * silu_f(z[(size_t)b * kVDim + (size_t)vh * kHd + c]);
        }
    }
}

template <int SPLIT, bool FUSED>
cudaError_t launch_t(cudaStream_t st, int b0, int nb, const qm_dn_params* p, qm_dn_state* s,
                     const float* qkv, const float* a, const float* b, float* y, const float* z,
                     float* out, int slot_w) {
    dim3 grid(s->nvh * SPLIT, nb);
    if (FUSED && SPLIT > 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = SPLIT;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, dn_decode_kernel<SPLIT, FUSED>, qkv, a, b, p->conv_w,
                                  p->a_log, p->dt_bias, p->norm_gamma, s->s, s->conv, slot_w, y,
                                  z, out, s->vh_lo, s->nvh, b0);
    }
    dn_decode_kernel<SPLIT, FUSED><<<grid, 256, 0, st>>>(qkv, a, b, p->conv_w, p->a_log,
                                                         p->dt_bias, p->norm_gamma, s->s, s->conv,
                                                         slot_w, y, z, out, s->vh_lo, s->nvh, b0);
    return cudaGetLastError();
}

}  // namespace

int dn_decode_split_for(int units, int num_sms) {
    if (units >= num_sms) return 1;
    if (units * 2 >= num_sms) return 2;
    return 4;
}

cudaError_t launch_dn_decode(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                             const float* a, const float* b, float* y, const float* z, float* out,
                             int b0, int nb) {
    const int B = nb < 0 ? st->batch : nb;
    const int slot_w = (int)(st->conv_pos & 3);
    const int split = dn_decode_split_for(B * st->nvh, ctx->num_sms);
    const bool fused = (z != nullptr);
    cudaError_t e;
    TimedLaunch tl(ctx, "dn_decode");
    if (split == 1)
        e = fused ? launch_t<1, true>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w)
                  : launch_t<1, false>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w);
    else if (split == 2)
        e = fused ? launch_t<2, true>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w)
                  : launch_t<2, false>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w);
    else
        e = fused ? launch_t<4, true>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w)
                  : launch_t<4, false>(ctx->stream, b0, B, p, st, qkv, a, b, y, z, out, slot_w);
    if (e == cudaSuccess) ctx->launches += 1;
    return e;
}

}  // namespace qm
