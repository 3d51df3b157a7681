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
//
// When the batch covers the GPU (B * heads >= SMs) a staged variant runs
// instead: each head's 64 KB state arrives in shared memory by bulk copy
// (issued first, so the conv/norm prologue overlaps it) and rows are read
// from there pass by pass, which keeps registers low enough for three CTAs
// per SM, i.e. three heads' states in flight per SM instead of two.
// Measured at batch 64: 5.17 TB/s against 5.09 for the register version; a
// persistent variant with three buffers per CTA (loads two heads ahead) ran
// 4.33 TB/s (one CTA per SM cannot hide the per-head chain), and writing the
// updated head back with one bulk store 4.92 TB/s.
#include <cooperative_groups.h>

#include "qm_internal.h"
#include "qm_ptx.cuh"

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

// ---------------------------------------------------------------------------
// Staged variant: heads item = blockIdx.x + k * gridDim.x (item = sequence *
// nvh + head), the same per-row arithmetic as dn_decode_kernel<1, FUSED>.
// With NB buffers a CTA requests up to NB heads ahead; the library launches
// one CTA per head (NB = 1, three CTAs per SM).
// ---------------------------------------------------------------------------
constexpr int kHeadBytes = kHd * kHd * 4;  // one head's state: 64 KB

// Raw per-thread inputs of one head: threads < 128 own q and k channel tid,
// threads >= 128 own v channel tid - 128; thread 255 also the gate inputs.
struct DnHeadIn {
    float x0, x1;            // q, k (or v, 0) of this token
    float r[6];              // history slots s0, s1, s2 of the same channels
    float4 w0, w1;           // conv taps
    float a, bb, alog, dtb;  // gate inputs (thread 255)
    float zv;                // z of the gated epilogue (threads < 128)
};

__device__ __forceinline__ void dn_fetch_head(DnHeadIn& in, const float* __restrict__ qkv,
                                              const float* __restrict__ a_in,
                                              const float* __restrict__ b_in,
                                              const float* __restrict__ conv_w,
                                              const float* __restrict__ a_log,
                                              const float* __restrict__ dt_bias,
                                              const float* __restrict__ conv,
                                              const float* __restrict__ z, int b, int vh,
                                              int s0, int s1, int s2, int tid) {
    const float* x = qkv + (size_t)b * kQKVDim;
    const float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
    if (tid < kHd) {
        const int chq = (vh >> 1) * kHd + tid, chk = kQDim + (vh >> 1) * kHd + tid;
        in.w0 = reinterpret_cast<const float4*>(conv_w)[chq];
        in.w1 = reinterpret_cast<const float4*>(conv_w)[chk];
        in.x0 = x[chq];
        in.x1 = x[chk];
        in.r[0] = ring[s0 * kQKVDim + chq];
        in.r[1] = ring[s1 * kQKVDim + chq];
        in.r[2] = ring[s2 * kQKVDim + chq];
        in.r[3] = ring[s0 * kQKVDim + chk];
        in.r[4] = ring[s1 * kQKVDim + chk];
        in.r[5] = ring[s2 * kQKVDim + chk];
        // fetched with the other inputs so its latency hides behind this head's work
        in.zv = z ? z[(size_t)b * kVDim + (size_t)vh * kHd + tid] : 0.f;
    } else {
        const int chv = 2 * kQDim + vh * kHd + (tid - kHd);
        in.w0 = reinterpret_cast<const float4*>(conv_w)[chv];
        in.x0 = x[chv];
        in.r[0] = ring[s0 * kQKVDim + chv];
        in.r[1] = ring[s1 * kQKVDim + chv];
        in.r[2] = ring[s2 * kQKVDim + chv];
    }
    if (tid == 255) {
        in.a = a_in[b * kNumV + vh];
        in.bb = b_in[b * kNumV + vh];
        in.alog = a_log[vh];
        in.dtb = dt_bias[vh];
    }
}

// The inputs that differ between the two V heads of one QK head (v, its
// history and taps, z, the gates); q and k stay as fetched for the partner.
__device__ __forceinline__ void dn_fetch_vhead(DnHeadIn& in, const float* __restrict__ qkv,
                                               const float* __restrict__ a_in,
                                               const float* __restrict__ b_in,
                                               const float* __restrict__ conv_w,
                                               const float* __restrict__ a_log,
                                               const float* __restrict__ dt_bias,
                                               const float* __restrict__ conv,
                                               const float* __restrict__ z, int b, int vh, int s0,
                                               int s1, int s2, int tid) {
    const float* x = qkv + (size_t)b * kQKVDim;
    const float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
    if (tid < kHd) {
        in.zv = z ? z[(size_t)b * kVDim + (size_t)vh * kHd + tid] : 0.f;
    } else {
        const int chv = 2 * kQDim + vh * kHd + (tid - kHd);
        in.w0 = reinterpret_cast<const float4*>(conv_w)[chv];
        in.x0 = x[chv];
        in.r[0] = ring[s0 * kQKVDim + chv];
        in.r[1] = ring[s1 * kQKVDim + chv];
        in.r[2] = ring[s2 * kQKVDim + chv];
    }
    if (tid == 255) {
        in.a = a_in[b * kNumV + vh];
        in.bb = b_in[b * kNumV + vh];
        in.alog = a_log[vh];
        in.dtb = dt_bias[vh];
    }
}

// NB shared buffers per CTA; MINB CTAs per SM.  PAIR: CTA c takes the two V
// heads 2c, 2c+1 of the item list (the two V heads of one QK head of one
// sequence) one after the other and fetches q and k once for both — used when
// the inputs are read from host memory over PCIe, where each byte counts.
template <bool FUSED, int NB, int MINB, bool PAIR = false>
__global__ void __launch_bounds__(256, MINB)
dn_decode_stream(const float* __restrict__ qkv, const float* __restrict__ a_in,
                 const float* __restrict__ b_in, const float* __restrict__ conv_w,
                 const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                 const float* __restrict__ norm_gamma, float* __restrict__ S,
                 float* __restrict__ conv, int slot_w, float* __restrict__ y,
                 const float* __restrict__ z, float* __restrict__ out, int vh_lo, int nvh, int b0,
                 int n_items, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* buf0 = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ float s_qk[2][kHd];
    __shared__ float s_v[kHd];
    __shared__ float s_red[2][4];
    __shared__ float s_ab[2];
    __shared__ float s_y[kHd];
    __shared__ float s_wsq[8];
    __shared__ uint64_t full[NB];
    __shared__ int abort_flag_s;
    volatile int* abort_flag = &abort_flag_s;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lane8 = lane & 7, rsub = lane >> 3;
    const int G = gridDim.x;
    const int s0 = (slot_w + 1) & 3, s1 = (slot_w + 2) & 3, s2 = (slot_w + 3) & 3;
    // heads of this CTA and the item of its k-th head
    const int nk = PAIR ? 2 : (n_items - (int)blockIdx.x + G - 1) / G;
    auto item_of = [&](int k) { return PAIR ? 2 * (int)blockIdx.x + k : (int)blockIdx.x + k * G; };

    if (tid == 0) {
        for (int i = 0; i < NB; i++) mbar_init(smem_u32(&full[i]), 1);
        abort_flag_s = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // thread 0: the last head whose state was requested into each buffer and
    // not yet waited for (drained on the way out of an aborted CTA)
    int pending[NB];
#pragma unroll
    for (int i = 0; i < NB; i++) pending[i] = -1;
    auto issue = [&](int k) {  // state of this CTA's k-th head into buffer k % NB
        const int item = item_of(k);
        const int buf = k % NB;
        const int b = b0 + item / nvh, lh = item % nvh;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(S + ((size_t)b * nvh + lh) * kHd * kHd);
        const uint32_t fb = smem_u32(&full[buf]);
        mbar_arrive_expect_tx(fb, kHeadBytes);
        for (int part = 0; part < 4; part++)
            bulk_load(smem_u32(buf0 + buf * kHeadBytes + part * (kHeadBytes / 4)), src + part * (kHeadBytes / 4),
                      kHeadBytes / 4, fb);
        pending[buf] = k;
    };
    if (tid == 0)
        for (int k = 0; k < NB && k < nk; k++) issue(k);

    DnHeadIn cur, nxt;
    if (nk > 0) {
        const int item = item_of(0), b = b0 + item / nvh, vh = vh_lo + item % nvh;
        dn_fetch_head(nxt, qkv, a_in, b_in, conv_w, a_log, dt_bias, conv, z, b, vh, s0, s1, s2, tid);
    }
    bool ok = true;
    for (int k = 0; k < nk && ok; k++) {
        const int item = item_of(k);
        const int b = b0 + item / nvh, lh = item % nvh, vh = vh_lo + lh;
        const int buf = k % NB;
        cur = nxt;
        if (k + 1 < nk) {  // the next head's inputs, in flight during this one
            const int it2 = item_of(k + 1), b2 = b0 + it2 / nvh, vh2 = vh_lo + it2 % nvh;
            if (PAIR)  // the partner V head: same q and k
                dn_fetch_vhead(nxt, qkv, a_in, b_in, conv_w, a_log, dt_bias, conv, z, b2, vh2, s0, s1, s2, tid);
            else
                dn_fetch_head(nxt, qkv, a_in, b_in, conv_w, a_log, dt_bias, conv, z, b2, vh2, s0, s1, s2, tid);
        }

        // ---- prologue: conv1d(k=4) + SiLU + L2 norm (gemv.rs:744-785) ----
        float* ring = conv + (size_t)b * kConvSlots * kQKVDim;
        float qv = 0.f, kv = 0.f;
        if (tid < kHd) {
            float cq = cur.r[0] * cur.w0.x;
            cq += cur.r[1] * cur.w0.y;
            cq += cur.r[2] * cur.w0.z;
            cq += cur.x0 * cur.w0.w;
            float ck = cur.r[3] * cur.w1.x;
            ck += cur.r[4] * cur.w1.y;
            ck += cur.r[5] * cur.w1.z;
            ck += cur.x1 * cur.w1.w;
            qv = silu_f(cq);
            kv = silu_f(ck);
            if ((vh & 1) == 0) {  // one head per QK head advances its history
                const int qk = vh >> 1;
                ring[slot_w * kQKVDim + qk * kHd + tid] = cur.x0;
                ring[slot_w * kQKVDim + kQDim + qk * kHd + tid] = cur.x1;
            }
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
        } else {
            const int c = tid - kHd;
            float cv = cur.r[0] * cur.w0.x;
            cv += cur.r[1] * cur.w0.y;
            cv += cur.r[2] * cur.w0.z;
            cv += cur.x0 * cur.w0.w;
            s_v[c] = silu_f(cv);
            ring[slot_w * kQKVDim + 2 * kQDim + vh * kHd + c] = cur.x0;
        }
        if (tid == 255) {  // alpha/beta (gemv.rs:791-800)
            const float a_exp = __expf(cur.alog);
            const float sp = softplus_f(cur.a + cur.dtb);
            s_ab[0] = __expf(-a_exp * sp);
            s_ab[1] = 1.0f / (1.0f + __expf(-cur.bb));
        }
        __syncthreads();
        if (tid < kHd) {  // l2_normalize (gemv.rs:641-649), q *= 1/sqrt(128) (784)
            const float nq = sqrtf(s_red[0][0] + s_red[0][1] + s_red[0][2] + s_red[0][3]);
            const float nk2 = sqrtf(s_red[1][0] + s_red[1][1] + s_red[1][2] + s_red[1][3]);
            if (nq > 1e-12f) qv *= 1.0f / nq;
            if (nk2 > 1e-12f) kv *= 1.0f / nk2;
            s_qk[0][tid] = qv * 0.08838834764831845f;
            s_qk[1][tid] = kv;
        }
        const bool w = mbar_wait_bounded(smem_u32(&full[buf]), (k / NB) & 1, abort_flag, err);
        if (tid == 0 && w) pending[buf] = -1;
        ok = __syncthreads_and(w) != 0;
        if (!ok) break;

        // ---- fused state update (simd.rs:304-361 in one pass), rows from shared ----
        const float alpha = s_ab[0], beta = s_ab[1];
        float4 kr[4], qr[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            kr[j] = reinterpret_cast<const float4*>(s_qk[1])[j * 8 + lane8];
            qr[j] = reinterpret_cast<const float4*>(s_qk[0])[j * 8 + lane8];
        }
        const float* Sb = reinterpret_cast<const float*>(buf0 + buf * kHeadBytes);
        float* Sh = S + ((size_t)b * nvh + lh) * kHd * kHd;
        float* yb = y ? y + ((size_t)b * nvh + lh) * kHd : nullptr;
        float sq_part = 0.f;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int r = p * 32 + warp * 4 + rsub;
            float4 sr[4];
#pragma unroll
            for (int j = 0; j < 4; j++) sr[j] = reinterpret_cast<const float4*>(Sb + (size_t)r * kHd)[j * 8 + lane8];
            const float vr = s_v[r];
            float pk0 = 0.f, pk1 = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float4& st = sr[j];
                st.x *= alpha; st.y *= alpha; st.z *= alpha; st.w *= alpha;
                pk0 = fmaf(st.x, kr[j].x, pk0);
                pk1 = fmaf(st.y, kr[j].y, pk1);
                pk0 = fmaf(st.z, kr[j].z, pk0);
                pk1 = fmaf(st.w, kr[j].w, pk1);
            }
            float pk = pk0 + pk1;
            pk += __shfl_xor_sync(0xffffffffu, pk, 1);
            pk += __shfl_xor_sync(0xffffffffu, pk, 2);
            pk += __shfl_xor_sync(0xffffffffu, pk, 4);
            const float delta = beta * (vr - pk);
            float py0 = 0.f, py1 = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float4& st = sr[j];
                st.x = fmaf(delta, kr[j].x, st.x);
                st.y = fmaf(delta, kr[j].y, st.y);
                st.z = fmaf(delta, kr[j].z, st.z);
                st.w = fmaf(delta, kr[j].w, st.w);
                py0 = fmaf(st.x, qr[j].x, py0);
                py1 = fmaf(st.y, qr[j].y, py1);
                py0 = fmaf(st.z, qr[j].z, py0);
                py1 = fmaf(st.w, qr[j].w, py1);
            }
            float yr = py0 + py1;
            yr += __shfl_xor_sync(0xffffffffu, yr, 1);
            yr += __shfl_xor_sync(0xffffffffu, yr, 2);
            yr += __shfl_xor_sync(0xffffffffu, yr, 4);
            float4* row = reinterpret_cast<float4*>(Sh + (size_t)r * kHd);
#pragma unroll
            for (int j = 0; j < 4; j++) row[j * 8 + lane8] = sr[j];
            if (lane8 == 0) {
                if (yb) yb[r] = yr;
                if (FUSED) {
                    s_y[r] = yr;
                    sq_part += yr * yr;
                }
            }
        }

        // ---- optional epilogue: RMSNorm(y)*gamma*SiLU(z) (gemv.rs:864-883) ----
        if constexpr (FUSED) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sq_part += __shfl_xor_sync(0xffffffffu, sq_part, o);
            if (lane == 0) s_wsq[warp] = sq_part;
            __syncthreads();
            float total = 0.f;
#pragma unroll
            for (int wi = 0; wi < 8; wi++) total += s_wsq[wi];
            const float inv_rms = 1.0f / sqrtf(total * (1.0f / kHd) + 1e-6f);
            if (tid < kHd) {
                const float yn = s_y[tid] * inv_rms * norm_gamma[tid];
                out[((size_t)b * nvh + lh) * kHd + tid] = yn * silu_f(cur.zv);
            }
        }
        __syncthreads();  // the buffer, s_qk, s_v, s_y are free again
        if (tid == 0 && k + NB < nk) issue(k + NB);
    }
    // do not leave while copies this CTA issued may still land
    if (tid == 0)
        for (int i = 0; i < NB; i++)
            if (pending[i] >= 0) mbar_drain(smem_u32(&full[i]), (pending[i] / NB) & 1, err);
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

constexpr int kStreamNB = 1, kStreamMinB = 3;  // one buffer per CTA, three CTAs per SM
constexpr int kStreamSmem = kStreamNB * kHeadBytes + 1024;

template <bool FUSED, bool PAIR>
cudaError_t launch_stream(qm_ctx* ctx, int b0, int nb, const qm_dn_params* p, qm_dn_state* s,
                          const float* qkv, const float* a, const float* b, float* y,
                          const float* z, float* out, int slot_w) {
    auto kern = dn_decode_stream<FUSED, kStreamNB, kStreamMinB, PAIR>;
    static std::atomic<uint64_t> attr_set{0};  // one per template instance
    const cudaError_t ea = set_smem_once(attr_set, ctx->device, kern, kStreamSmem);
    if (ea != cudaSuccess) return ea;
    const int n_items = nb * s->nvh;
    const int grid = PAIR ? n_items / 2 : n_items;  // one CTA per head (per V-head pair)
    kern<<<grid, 256, kStreamSmem, ctx->stream>>>(
        qkv, a, b, p->conv_w, p->a_log, p->dt_bias, p->norm_gamma, s->s, s->conv, slot_w, y, z, out,
        s->vh_lo, s->nvh, b0, n_items, ctx->d_err);
    return cudaGetLastError();
}

int dn_decode_split_for(int units, int num_sms) {
    if (units >= num_sms) return 1;
    if (units * 2 >= num_sms) return 2;
    return 4;
}

cudaError_t launch_dn_decode(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, const float* qkv,
                             const float* a, const float* b, float* y, const float* z, float* out,
                             int b0, int nb, bool pair) {
    const int B = nb < 0 ? st->batch : nb;
    const int slot_w = (int)(st->conv_pos & 3);
    const int split = dn_decode_split_for(B * st->nvh, ctx->num_sms);
    const bool fused = (z != nullptr);
    cudaError_t e;
    TimedLaunch tl(ctx, "dn_decode");
    if (split == 1 && pair)  // inputs in host memory: q and k fetched once per V-head pair
        e = fused ? launch_stream<true, true>(ctx, b0, B, p, st, qkv, a, b, y, z, out, slot_w)
                  : launch_stream<false, true>(ctx, b0, B, p, st, qkv, a, b, y, z, out, slot_w);
    else if (split == 1)  // the batch covers the GPU: staged CTAs, three per SM
        e = fused ? launch_stream<true, false>(ctx, b0, B, p, st, qkv, a, b, y, z, out, slot_w)
                  : launch_stream<false, false>(ctx, b0, B, p, st, qkv, a, b, y, z, out, slot_w);
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
