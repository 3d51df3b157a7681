// The decode loop's tail next to the mixer stack: lm_head over the tied
// embedding rows, the logit penalties and top-k / top-p sampling.  The
// reference runs all three on the CPU every token (src/gemv.rs:662-711,
// src/generate.rs:58-83, 185-198, 334-384).
//
// qm_rows_kernel<Q4, BT>: y[b][v] = x[b] . E[v] for weights stored one row
// per output (QM_W_F16_ROWS: f16 [n][k]; QM_W_Q4_ROWS: packed [n][k/2] and
// f16 scales [n][k/32], groups of 32 along k).  HBM-bound: every weight byte
// is read once per call.  A warp takes 4 rows at a time; lane l the 16-byte
// chunks l, l+32, l+64, ... of each row (one Q4 group or 8 f16 values), all
// of them in flight at once.  x is staged in shared memory, chunk by chunk
// with 4 floats of padding (no bank conflicts), Q4 prescaled by
// 2^(-4 (j mod 4)) so the nibble trick of qm_gemv needs no shift (one LOP3,
// one FADD and one FFMA per weight); a lane's 4 rows reuse the x chunk it
// loaded.  Row sums are reduced across the warp in a fixed butterfly order.
// Q4 per weight is one AND and one FFMA: the nibble masked in place (no
// shift) read as a float is the denormal q 2^(4j - 149), x is staged
// prescaled by 2^(100 - 4j) (j = position mod 4), so their product is
// q x 2^-49 exactly; the group's sum is scaled back by 2^49 and the -8 of
// every nibble enters once a group as -8 sum(x), kept in the chunk's
// padding slot.  (Valid for |x| < 2^27; denormals are not flushed: no fast
// math.)
//
// qm_penalize_kernel: one CTA per sequence.  Repetition: the last
// min(len, 64) tokens; the first occurrence of each token id applies all of
// that id's divisions (positive logit) or multiplications in order.
// Presence: a bitmap of the vocabulary in shared memory; the thread whose
// atomic clear finds the bit set subtracts the penalty, so each seen token
// loses it exactly once.  Then the banned token (if any) becomes -inf.
//
// qm_sample_kernel: a cluster of 16 CTAs of 1024 threads per sequence, each
// over 1/16 of the vocabulary, each thread's 16 logits read once and kept
// as keys in registers (the histograms and candidate lists meet in
// distributed shared memory; rank 0 sorts and draws).  Greedy
// (temperature <= 0): the first index of the largest logit.  Otherwise the
// k largest logits in the reference's order (value descending, index
// ascending: its stable sort) are found with a radix select on the
// order-preserving 32-bit key (4 passes of 8 bits with one histogram per
// warp), collected (ties at the
// threshold: lowest indices first) and bitonic-sorted in shared memory; one
// thread then runs the reference's softmax / top-p / draw with its f32
// operations in its order.
// exp is (float)exp((double)x); the host's expf differs from it by one ulp
// for ~0.06 % of arguments, which moves a decision only when the draw lands
// within rounding of a cumulative boundary.
#include <cuda_fp16.h>

#include <atomic>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {
namespace {

constexpr int kRwThreads = 256;
constexpr int kRwRows = 4;  // rows per warp pass

template <bool Q4, int BT>
__global__ void __launch_bounds__(kRwThreads, 2)
qm_rows_kernel(const void* __restrict__ data, const uint16_t* __restrict__ scales, int k, int n,
               const float* __restrict__ x, float* __restrict__ y) {
    constexpr int NB = Q4 ? 3 : 4;   // chunks per lane per pass
    constexpr int CW = Q4 ? 32 : 8;  // weights per 16-byte chunk
    constexpr int XS = CW + 4;       // shared floats per chunk: lane l's float4 reads (chunk stride
                                     // 144 / 48 bytes) fall on distinct banks within each 8-lane phase
    extern __shared__ float xs[];    // [BT][C][XS]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = k / CW;
    for (int i = tid; i < BT * k; i += kRwThreads) {
        const int b = i / k, j = i % k;
        float v = x[i];
        if (Q4) v *= 1.2676506e30f / (float)(1u << (4 * (j & 3)));  // x 2^(100 - 4 (j mod 4)): exact
        xs[(b * C + j / CW) * XS + j % CW] = v;
    }
    if (Q4) {  // each chunk's plain sum of x in its padding slot (for the -8 of every nibble)
        for (int i = tid; i < BT * C; i += kRwThreads) {
            const float* xc = x + (size_t)(i / C) * k + (size_t)(i % C) * CW;
            float t = 0.f;
            for (int j = 0; j < CW; j++) t += xc[j];
            xs[i * XS + CW] = t;
        }
    }
    __syncthreads();
    const int groups = (n + kRwRows - 1) / kRwRows;
    const int nwarps = gridDim.x * (kRwThreads / 32);
    for (int grp = blockIdx.x * (kRwThreads / 32) + warp; grp < groups; grp += nwarps) {
        const int v0 = grp * kRwRows;
        float acc[BT][kRwRows];
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int rr = 0; rr < kRwRows; rr++) acc[b][rr] = 0.f;
        for (int cb = 0; cb < C; cb += 32 * NB) {
            uint4 w[kRwRows][NB];
            uint32_t s[kRwRows][Q4 ? NB : 1];
#pragma unroll
            for (int rr = 0; rr < kRwRows; rr++)
#pragma unroll
                for (int i = 0; i < NB; i++) {
                    const int c = cb + 32 * i + lane;
                    const int row = v0 + rr;
                    const bool ok = c < C && row < n;
                    if (Q4) {
                        const uint8_t* p = static_cast<const uint8_t*>(data) + (size_t)row * (k / 2) + (size_t)c * 16;
                        w[rr][i] = ok ? __ldcs(reinterpret_cast<const uint4*>(p))
                                      : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
                        s[rr][Q4 ? i : 0] = ok ? __ldcs(reinterpret_cast<const unsigned short*>(scales + (size_t)row * (k / 32) + c)) : 0u;
                    } else {
                        const uint16_t* p = static_cast<const uint16_t*>(data) + (size_t)row * k + (size_t)c * 8;
                        w[rr][i] = ok ? __ldcs(reinterpret_cast<const uint4*>(p)) : make_uint4(0u, 0u, 0u, 0u);
                    }
                }
#pragma unroll
            for (int i = 0; i < NB; i++) {
                const int c = cb + 32 * i + lane;
                if (c >= C) break;
#pragma unroll
                for (int b = 0; b < BT; b++) {
                    float xv[CW];
#pragma unroll
                    for (int q = 0; q < CW / 4; q++) {
                        const float4 f = *reinterpret_cast<const float4*>(&xs[(b * C + c) * XS + 4 * q]);
                        xv[4 * q] = f.x;
                        xv[4 * q + 1] = f.y;
                        xv[4 * q + 2] = f.z;
                        xv[4 * q + 3] = f.w;
                    }
#pragma unroll
                    for (int rr = 0; rr < kRwRows; rr++) {
                        const uint32_t ww[4] = {w[rr][i].x, w[rr][i].y, w[rr][i].z, w[rr][i].w};
                        if (Q4) {
                            // the nibble masked in place is the denormal q 2^(4j-149); times the
                            // prescaled x it is q x 2^-49 exactly, whatever j
                            // one chain of column pairs per word (packed f32x2 FMA: two products an
                            // instruction), 4 independent chains
                            float2 part[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                              make_float2(0.f, 0.f)};
#pragma unroll
                            for (int wd = 0; wd < 4; wd++) {
                                const uint32_t halves[2] = {ww[wd], ww[wd] >> 16};
#pragma unroll
                                for (int hh = 0; hh < 2; hh++)
#pragma unroll
                                    for (int jn = 0; jn < 4; jn += 2) {
                                        const int e = 8 * wd + 4 * hh + jn;
                                        part[wd] = __ffma2_rn(
                                            make_float2(__uint_as_float(halves[hh] & (0xFu << (4 * jn))),
                                                        __uint_as_float(halves[hh] & (0xF0u << (4 * jn)))),
                                            make_float2(xv[e], xv[e + 1]), part[wd]);
                                    }
                            }
                            const float qx = (((part[0].x + part[0].y) + (part[1].x + part[1].y)) +
                                              ((part[2].x + part[2].y) + (part[3].x + part[3].y))) *
                                             562949953421312.0f;  // 2^49
                            const float xsum = xs[(b * C + c) * XS + CW];
                            const float sc = __half2float(__ushort_as_half((uint16_t)s[rr][Q4 ? i : 0]));
                            acc[b][rr] = fmaf(sc, fmaf(-8.0f, xsum, qx), acc[b][rr]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[q]));
                                acc[b][rr] = fmaf(xv[2 * q], f.x, acc[b][rr]);
                                acc[b][rr] = fmaf(xv[2 * q + 1], f.y, acc[b][rr]);
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int rr = 0; rr < kRwRows; rr++) {
                float v = acc[b][rr];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (lane == rr && v0 + rr < n) y[(size_t)b * n + v0 + rr] = v;
            }
    }
}

template <bool Q4, int BT>
cudaError_t launch_rows_bt(qm_ctx* c, const qm_weight* w, const float* x, float* y) {
    auto kern = qm_rows_kernel<Q4, BT>;
    const int cw = Q4 ? 32 : 8;
    const size_t smem = (size_t)BT * (w->k / cw) * (cw + 4) * sizeof(float);
    static std::atomic<uint64_t> attr_set{0};
    const uint64_t bit = 1ull << (c->device & 63);
    if (!(attr_set.load() & bit)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    const int groups = (w->n + kRwRows - 1) / kRwRows;
    int grid = 2 * c->num_sms;
    const int need = (groups + kRwThreads / 32 - 1) / (kRwThreads / 32);
    if (grid > need) grid = need;
    kern<<<grid, kRwThreads, smem, c->stream>>>(w->data, static_cast<const uint16_t*>(w->scales), w->k, w->n, x, y);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// penalties
// ---------------------------------------------------------------------------
constexpr int kPenThreads = 256;

__global__ void __launch_bounds__(kPenThreads)
qm_penalize_kernel(float* logits, int vocab, const int* __restrict__ tokens, const int* __restrict__ lens,
                   int stride, float rep, float pres, int ban) {
    extern __shared__ uint32_t seen[];  // ceil(vocab / 32) words when pres > 0
    __shared__ int win[64];
    const int b = blockIdx.x, tid = threadIdx.x;
    float* lg = logits + (size_t)b * vocab;
    const int* tok = tokens + (size_t)b * stride;
    const int len = lens ? max(0, min(lens[b], stride)) : 0;  // a history never reads past its row
    if (rep > 1.0f && len > 0) {
        const int window = len < 64 ? len : 64;
        if (tid < window) win[tid] = tok[len - window + tid];
        __syncthreads();
        if (tid < window) {
            const int t = win[tid];
            bool first = true;
            for (int j = 0; j < tid; j++) first = first && win[j] != t;
            if (first && t >= 0 && t < vocab) {
                int cnt = 0;
                for (int j = tid; j < window; j++) cnt += win[j] == t;
                float l = lg[t];
                for (int q = 0; q < cnt; q++) l = l > 0.0f ? __fdiv_rn(l, rep) : __fmul_rn(l, rep);
                lg[t] = l;
            }
        }
        __syncthreads();
    }
    if (pres > 0.0f && len > 0) {
        const int words = (vocab + 31) / 32;
        for (int i = tid; i < words; i += kPenThreads) seen[i] = 0u;
        __syncthreads();
        for (int i = tid; i < len; i += kPenThreads) {
            const int t = tok[i];
            if (t >= 0 && t < vocab) atomicOr(&seen[t >> 5], 1u << (t & 31));
        }
        __syncthreads();
        for (int i = tid; i < len; i += kPenThreads) {
            const int t = tok[i];
            if (t >= 0 && t < vocab) {
                const uint32_t bitm = 1u << (t & 31);
                if (atomicAnd(&seen[t >> 5], ~bitm) & bitm) lg[t] = __fsub_rn(lg[t], pres);
            }
        }
        __syncthreads();
    }
    if (tid == 0 && ban >= 0 && ban < vocab) lg[ban] = -INFINITY;
}

// ---------------------------------------------------------------------------
// sampling
// ---------------------------------------------------------------------------
constexpr int kSmThreads = 1024;
constexpr int kSmWarps = kSmThreads / 32;
constexpr int kSmCluster = 16;  // CTAs per sequence, each over 1/16 of the vocabulary
constexpr int kSmPer = 16;      // keys a thread holds in registers: vocab <= 16 x 1024 x 16
constexpr int kSmMaxK = 4096;
constexpr int kSmBins = 256;  // 8-bit digits, one histogram per warp

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}
__device__ __forceinline__ uint32_t dsmem_u32(const void* p, uint32_t rank) {
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(mapa_shared(smem_u32(p), rank)));
    return v;
}
__device__ __forceinline__ unsigned long long dsmem_u64(const void* p, uint32_t rank) {
    unsigned long long v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(mapa_shared(smem_u32(p), rank)));
    return v;
}

// Dynamic shared memory: cand [kSmMaxK] u64 (rank 0: the gathered list),
// lcand [kSmMaxK] u64 (this CTA's candidates), prob [kSmMaxK] f32,
// whist [warps][kSmBins] u32.
__global__ void __launch_bounds__(kSmThreads, 1)
qm_sample_kernel(const float* __restrict__ logits, int vocab, float temperature, float top_p, int top_k,
                 const float* __restrict__ rdraw, int* __restrict__ ids) {
    extern __shared__ unsigned long long sm_u64[];
    unsigned long long* cand = sm_u64;
    unsigned long long* lcand = cand + kSmMaxK;
    float* prob = reinterpret_cast<float*>(lcand + kSmMaxK);
    uint32_t* whist = reinterpret_cast<uint32_t*>(prob + kSmMaxK);
    __shared__ uint32_t chist[kSmBins];  // this CTA's histogram (read by the whole cluster)
    __shared__ uint32_t ghist[kSmBins];  // the cluster's
    __shared__ float red_f[kSmWarps];
    __shared__ int red_i[kSmWarps];
    __shared__ float sh_cmax, sh_bv;
    __shared__ int sh_bi;
    __shared__ uint32_t sh_digit, sh_kleft, sh_eq_total, sh_ceq;
    __shared__ int sh_count;
    __shared__ int warp_eq[kSmWarps];
    const uint32_t rank = cluster_ctarank();
    const int b = blockIdx.x / kSmCluster, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float* lg = logits + (size_t)b * vocab;
    const int per = (vocab + kSmCluster - 1) / kSmCluster;
    const int lo = (int)rank * per, hi = min(vocab, lo + per);

    if (temperature <= 0.0f) {  // greedy: the first index of the largest value (NaN never wins)
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int i = lo + tid; i < hi; i += kSmThreads) {
            const float v = lg[i];
            if (v > bv) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            red_f[warp] = bv;
            red_i[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float fv = -INFINITY;
            int fi = 0x7FFFFFFF;
            for (int w = 0; w < kSmWarps; w++)
                if (red_f[w] > fv || (red_f[w] == fv && red_i[w] < fi)) {
                    fv = red_f[w];
                    fi = red_i[w];
                }
            sh_bv = fv;
            sh_bi = fi;
        }
        cluster_sync_all();
        if (rank == 0 && tid == 0) {
            float fv = -INFINITY;
            int fi = 0x7FFFFFFF;
            for (uint32_t q = 0; q < kSmCluster; q++) {
                const float v = __uint_as_float(dsmem_u32(&sh_bv, q));
                const int i = (int)dsmem_u32(&sh_bi, q);
                if (v > fv || (v == fv && i < fi)) {
                    fv = v;
                    fi = i;
                }
            }
            ids[b] = fi == 0x7FFFFFFF ? 0 : fi;
        }
        cluster_sync_all();  // rank 0 has read every CTA's result before any leaves
        return;
    }
    const int k = top_k > 0 ? (top_k < vocab ? top_k : vocab) : vocab;

    // this thread's logits lo + tid + 1024 e, read once (all in flight) and
    // kept as order-preserving keys for every pass; the maximum on the way
    float mx = -INFINITY;
    uint32_t keys[kSmPer];
    const int nmine = hi - lo - tid > 0 ? (hi - lo - tid + kSmThreads - 1) / kSmThreads : 0;
    {
        float v[kSmPer];
#pragma unroll
        for (int e = 0; e < kSmPer; e++) v[e] = e < nmine ? lg[lo + tid + e * kSmThreads] : -INFINITY;
#pragma unroll
        for (int e = 0; e < kSmPer; e++) {
            mx = fmaxf(mx, v[e]);
            keys[e] = order_key(v[e]);
        }
    }

    // radix select of the k-th largest key, 8 bits a pass from the top.  Each
    // warp counts its elements into its own histogram; the CTA adds its 32,
    // the cluster adds its 16 CTAs' (every CTA the same sums, so every CTA
    // picks the same digit).
    uint32_t prefix = 0u, pmask = 0u, kleft = (uint32_t)k;
    uint32_t* myhist = whist + warp * kSmBins;
    for (int pass = 0; pass < 4; pass++) {
        const int sh = 24 - 8 * pass;
        for (int i = tid; i < kSmWarps * kSmBins; i += kSmThreads) whist[i] = 0u;
        __syncthreads();
#pragma unroll
        for (int e = 0; e < kSmPer; e++)
            if (e < nmine && (keys[e] & pmask) == prefix) atomicAdd(&myhist[(keys[e] >> sh) & 255u], 1u);
        if (pass == 0) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            if (lane == 0) red_f[warp] = mx;
        }
        __syncthreads();
        if (tid < kSmBins) {
            uint32_t tot = 0u;
            for (int w = 0; w < kSmWarps; w++) tot += whist[w * kSmBins + tid];
            chist[tid] = tot;
        }
        if (pass == 0 && tid == 0) {
            float m = red_f[0];
            for (int w = 1; w < kSmWarps; w++) m = fmaxf(m, red_f[w]);
            sh_cmax = m;
        }
        cluster_sync_all();  // every CTA's histogram (and maximum) is complete
        if (tid < kSmBins) {  // all 16 remote loads in flight, then the adds in rank order
            uint32_t h8[kSmCluster];
#pragma unroll
            for (int q = 0; q < kSmCluster; q++) h8[q] = dsmem_u32(&chist[tid], (uint32_t)q);
            uint32_t tot = 0u;
#pragma unroll
            for (int q = 0; q < kSmCluster; q++) tot += h8[q];
            ghist[tid] = tot;
        }
        if (pass == 0 && tid == kSmBins) {
            float m8[kSmCluster];
#pragma unroll
            for (int q = 0; q < kSmCluster; q++) m8[q] = __uint_as_float(dsmem_u32(&sh_cmax, (uint32_t)q));
            float m = -INFINITY;
#pragma unroll
            for (int q = 0; q < kSmCluster; q++) m = fmaxf(m, m8[q]);
            red_f[0] = m;
        }
        __syncthreads();
        if (warp == 0) {  // the digit: the highest d with (count above d) < kleft <= (count from d up)
            // lane l owns bins [8 (31 - l), 8 (31 - l) + 8): lane 0 the top 8
            uint32_t c8[8], own = 0u;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                c8[e] = ghist[8 * (31 - lane) + 7 - e];  // e = 0: this lane's highest bin
                own += c8[e];
            }
            uint32_t above = own;  // inclusive prefix over lanes 0..lane (bins from the top)
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t o = __shfl_up_sync(0xffffffffu, above, off);
                if (lane >= off) above += o;
            }
            above -= own;  // count in the bins above this lane's
            const bool mine = above < kleft && above + own >= kleft;
            const uint32_t who = __ballot_sync(0xffffffffu, mine);
            if (who == 0u) {  // cannot happen while kleft <= the matching count; take bin 0
                if (lane == 31) {
                    sh_digit = 0u;
                    sh_kleft = kleft - (above + own - c8[7]);
                    if (pass == 3) sh_eq_total = c8[7];
                }
            } else if (lane == __ffs(who) - 1) {
                uint32_t cum = above;
                int e = 0;
                for (; e < 7; e++) {
                    if (cum + c8[e] >= kleft) break;
                    cum += c8[e];
                }
                sh_digit = (uint32_t)(8 * (31 - lane) + 7 - e);
                sh_kleft = kleft - cum;
                if (pass == 3) sh_eq_total = c8[e];
            }
        }
        __syncthreads();
        if (pass == 0) mx = red_f[0];
        prefix |= sh_digit << sh;
        pmask |= 255u << sh;
        kleft = sh_kleft;
        cluster_sync_all();  // every CTA has read the others' histograms before they are reused
    }
    const uint32_t T = prefix;    // the k-th largest key
    const uint32_t k_eq = kleft;  // how many keys equal to T are taken
    const bool all_eq = sh_eq_total == k_eq;
    if (tid == 0) sh_count = 0;
    __syncthreads();
    if (all_eq) {  // no tie straddles the cut: every key >= T is a candidate
#pragma unroll
        for (int e = 0; e < kSmPer; e++) {
            const uint32_t i = (uint32_t)(lo + tid + e * kSmThreads);
            if (e < nmine && keys[e] >= T) lcand[atomicAdd(&sh_count, 1)] = ((unsigned long long)keys[e] << 32) | (0xFFFFFFFFu - i);
        }
    } else {  // keys > T, then the k_eq lowest-index keys == T: warp ranges, then CTAs, in index order
        const int span = hi > lo ? hi - lo : 0;
        const int wper = (((span + kSmWarps - 1) / kSmWarps) + 31) & ~31;
        const int wlo = lo + warp * wper, whi = min(hi, wlo + wper);
        int cnt = 0;
        for (int i = wlo + lane; i < whi; i += 32) {
            const uint32_t key = order_key(lg[i]);
            cnt += key == T;
            if (key > T) lcand[atomicAdd(&sh_count, 1)] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, off);
        if (lane == 0) warp_eq[warp] = cnt;
        __syncthreads();
        if (tid == 0) {
            uint32_t t = 0u;
            for (int w = 0; w < kSmWarps; w++) t += (uint32_t)warp_eq[w];
            sh_ceq = t;
        }
        cluster_sync_all();  // every CTA's count of keys == T
        uint32_t rankq = 0u;
        for (uint32_t q = 0; q < rank; q++) rankq += dsmem_u32(&sh_ceq, q);
        for (int w = 0; w < warp; w++) rankq += (uint32_t)warp_eq[w];
        for (int i0 = wlo; i0 < whi; i0 += 32) {
            const int i = i0 + lane;
            const bool eq = i < whi && order_key(lg[i]) == T;
            const uint32_t bal = __ballot_sync(0xffffffffu, eq);
            const uint32_t my = rankq + __popc(bal & ((1u << lane) - 1u));
            if (eq && my < k_eq) lcand[atomicAdd(&sh_count, 1)] = ((unsigned long long)T << 32) | (0xFFFFFFFFu - (uint32_t)i);
            rankq += __popc(bal);
        }
    }
    cluster_sync_all();  // every CTA's candidate list is complete
    if (rank == 0) {     // gather the k candidates
        int base = 0;
        for (uint32_t q = 0; q < kSmCluster; q++) {
            const int cq = (int)dsmem_u32(&sh_count, q);
            for (int i = tid; i < cq; i += kSmThreads) cand[base + i] = dsmem_u64(&lcand[i], q);
            base += cq;
        }
    }
    cluster_sync_all();  // rank 0 has read every list before any CTA leaves
    if (rank != 0) return;
    // bitonic sort, descending by (key, -index): value descending, index ascending
    int P = 1;
    while (P < k) P <<= 1;
    for (int i = k + tid; i < P; i += kSmThreads) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += kSmThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const unsigned long long a = cand[i], c2 = cand[j];
                    const bool desc = (i & size) == 0;
                    if (desc ? (a < c2) : (a > c2)) {
                        cand[i] = c2;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    // the reference's softmax / top-p / draw over the k sorted candidates
    const float inv_temp = __fdiv_rn(1.0f, temperature);
    for (int i = tid; i < k; i += kSmThreads) {
        const float v = key_value((uint32_t)(cand[i] >> 32));
        prob[i] = (float)exp((double)__fmul_rn(__fsub_rn(v, mx), inv_temp));
    }
    __syncthreads();
    if (tid == 0) {
        const int id0 = (int)(0xFFFFFFFFu - (uint32_t)(cand[0] & 0xFFFFFFFFull));
        float sum = 0.0f;
        for (int i = 0; i < k; i++) sum = __fadd_rn(sum, prob[i]);
        int out = id0;
        if (sum > 0.0f) {
            const float inv = __fdiv_rn(1.0f, sum);
            float cum = 0.0f;
            int cutoff = k;
            for (int i = 0; i < k; i++) {
                prob[i] = __fmul_rn(prob[i], inv);
                cum = __fadd_rn(cum, prob[i]);
                if (cum >= top_p) {
                    cutoff = i + 1;
                    break;
                }
            }
            float total = 0.0f;
            for (int i = 0; i < cutoff; i++) total = __fadd_rn(total, prob[i]);
            if (total > 0.0f) {
                const float rv = __fmul_rn(rdraw[b], total);
                float acc = 0.0f;
                for (int i = 0; i < cutoff; i++) {
                    acc = __fadd_rn(acc, prob[i]);
                    if (acc >= rv) {
                        out = (int)(0xFFFFFFFFu - (uint32_t)(cand[i] & 0xFFFFFFFFull));
                        break;
                    }
                }
            }
        }
        ids[b] = out;
    }
}

}  // namespace

int gemv_rows(qm_ctx* c, const qm_weight* w, int batch, const float* x, float* y) {
    const bool q4 = w->kind == QM_W_Q4_ROWS;
    if (q4) {
        if (!w->scales) return set_error(c, QM_E_ARG, "Q4 weights need scales");
        if (w->k % 32) return set_error(c, QM_E_SHAPE, "Q4 rows need k % 32 == 0 (groups of 32 along k)");
        if (((uintptr_t)w->data & 15) || ((uintptr_t)w->scales & 1))
            return set_error(c, QM_E_ARG, "Q4 data must be 16-byte and scales 2-byte aligned");
    } else {
        if (w->k % 8) return set_error(c, QM_E_SHAPE, "F16 rows need k % 8 == 0");
        if ((uintptr_t)w->data & 15) return set_error(c, QM_E_ARG, "F16 data must be 16-byte aligned");
    }
    if ((size_t)2 * (w->k / 8) * 12 * sizeof(float) > 200 * 1024) return set_error(c, QM_E_SHAPE, "k too large");
    cudaSetDevice(c->device);
    TimedLaunch tl(c, "lm_head");
    const int bmax = q4 ? 1 : 2;  // Q4 at 2 sequences spills: one launch per sequence
    for (int b0 = 0; b0 < batch; b0 += bmax) {
        const int bt = batch - b0 < bmax ? batch - b0 : bmax;
        const float* xb = x + (size_t)b0 * w->k;
        float* yb = y + (size_t)b0 * w->n;
        cudaError_t e;
        if (q4) e = launch_rows_bt<true, 1>(c, w, xb, yb);
        else e = bt == 1 ? launch_rows_bt<false, 1>(c, w, xb, yb) : launch_rows_bt<false, 2>(c, w, xb, yb);
        if (e != cudaSuccess) return cuda_error(c, e, "qm_gemv rows launch");
        c->launches += 1;
    }
    return QM_OK;
}

}  // namespace qm

using namespace qm;

extern "C" int qm_logits_penalize(qm_ctx* c, float* logits, int batch, int vocab, const int* tokens,
                                  const int* lens, int stride, float repetition_penalty, float presence_penalty,
                                  int ban_token) {
    if (!c) return QM_E_ARG;
    if (!logits || batch < 1 || vocab < 1) return set_error(c, QM_E_ARG, "null logits or empty shape");
    const bool any_hist = repetition_penalty > 1.0f || presence_penalty > 0.0f;
    if (any_hist && (!tokens || !lens || stride < 0)) return set_error(c, QM_E_ARG, "penalties need tokens and lens");
    const size_t smem = presence_penalty > 0.0f ? (size_t)((vocab + 31) / 32) * 4 : 0;
    if (smem > 200 * 1024) return set_error(c, QM_E_SHAPE, "vocabulary too large for the presence bitmap");
    if (!any_hist && ban_token < 0) return QM_OK;
    cudaSetDevice(c->device);
    static std::atomic<uint64_t> attr_set{0};
    const uint64_t bit = 1ull << (c->device & 63);
    if (!(attr_set.load() & bit)) {
        const cudaError_t e =
            cudaFuncSetAttribute(qm_penalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return cuda_error(c, e, "qm_logits_penalize setup");
        attr_set.fetch_or(bit);
    }
    TimedLaunch tl(c, "penalize");
    qm_penalize_kernel<<<batch, kPenThreads, smem, c->stream>>>(
        logits, vocab, any_hist ? tokens : nullptr, any_hist ? lens : nullptr, stride,
        any_hist ? repetition_penalty : 1.0f, any_hist ? presence_penalty : 0.0f, ban_token);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(c, e, "qm_logits_penalize launch");
    c->launches += 1;
    return QM_OK;
}

extern "C" int qm_sample(qm_ctx* c, const float* logits, int batch, int vocab, float temperature, float top_p,
                         int top_k, const float* r, int* ids) {
    if (!c) return QM_E_ARG;
    if (!logits || !ids || batch < 1 || vocab < 1) return set_error(c, QM_E_ARG, "null pointer or empty shape");
    if (!(temperature <= 0.0f)) {  // not greedy (as the reference tests it)
        if (!r) return set_error(c, QM_E_ARG, "sampling needs the draws r");
        if (vocab > kSmCluster * kSmThreads * kSmPer)
            return set_error(c, QM_E_UNSUPPORTED, "sampling holds at most 262,144 logits a sequence");
        const int k = top_k > 0 ? (top_k < vocab ? top_k : vocab) : vocab;
        if (k > kSmMaxK)
            return set_error(c, QM_E_UNSUPPORTED, "top_k must be in [1, 4096] (or the vocabulary at most 4096)");
    }
    cudaSetDevice(c->device);
    const size_t smem = (size_t)kSmMaxK * 16 + (size_t)kSmMaxK * 4 + (size_t)kSmWarps * kSmBins * 4;
    static std::atomic<uint64_t> attr_set{0};
    const uint64_t bit = 1ull << (c->device & 63);
    if (!(attr_set.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(qm_sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(qm_sample_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return cuda_error(c, e, "qm_sample setup");
        attr_set.fetch_or(bit);
    }
    TimedLaunch tl(c, "sample");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(batch * kSmCluster);
    cfg.blockDim = dim3(kSmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSmCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, qm_sample_kernel, logits, vocab, temperature, top_p, top_k, r, ids);
    if (e != cudaSuccess) return cuda_error(c, e, "qm_sample launch");
    c->launches += 1;
    return QM_OK;
}
