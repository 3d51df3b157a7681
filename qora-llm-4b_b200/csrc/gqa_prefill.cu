// GQA causal prefill on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces src/gemv.rs:1364-1444 (CPU: rayon over 16 heads, O(S^2 D) scalar
// loops) and src/gpu_inference.rs:690-766 (wgpu: materialises [16,S,S]
// scores with a -1e9 mask, 64 GiB per sequence at S = 32768).
//
// 1. gqa_prefill_prep  (B*T*4 CTAs): per token, QK-RMSNorm(1+g) + partial
//    RoPE at position t (gemv.rs:1388-1395).  The bf16 KV cache receives k
//    and v (gemv.rs:1397-1400: the prefill replaces the cache).  The attention
//    itself runs on fp16 operands — q*(1/16), the normed k and v converted
//    exactly from bf16 — written to a workspace: with the (1+gamma) norms the
//    scores have a std of ~4, and bf16's 8-bit mantissa on q and k alone
//    costs ~7e-2 of output error; fp16 (10 bits, same tensor-core rate) keeps
//    it near 1e-2.  fp16 holds these values with room to spare (|q/16| and
//    |k| stay below ~40, v below 65504 — larger v saturates).
// 2. gqa_prefill_attn  (one CTA per (sequence, head, 128-query tile)):
//    flash attention, causal, online softmax in base 2, 128-key tiles.
//      warp 0      TMA producer: one ring of 11 x 16 KB slots, filled in the
//                  order the consumers take them: the Q tile (4 slots), then
//                  K_0, and per tile j K_{j+1} ([128 keys x 64 dims] per slot)
//                  and V_j ([32 keys x 256 dims] per slot)
//      warp 1      TMEM owner + MMA issuer (one thread):
//                  S_j = Q K_j^T  (M=128, N=128, K=256: 16 x tcgen05.mma,
//                                  A = Q read from TMEM)
//                  O  += P_j V_j  (M=128, N=256, K=128:  8 x tcgen05.mma,
//                                  V read MN-major straight from its [pos][dim] boxes)
//                  in the order S_0, S_1, PV_0, S_2, PV_1, ...: while the
//                  softmax works on S_j, the tensor pipe runs S_{j+1} and PV_{j-1}
//      warps 2..9  softmax, two warps per TMEM lane quarter (64 score
//                  columns each): they first copy the Q tile from its ring
//                  slots into TMEM (so the S MMAs do not re-read 64 KB of
//                  shared memory per key tile), then per tile read S with
//                  tcgen05.ld, exchange the row max, write P to shared memory
//                  in the swizzled K-major layout the next MMA reads, and
//                  rescale the O accumulator in TMEM only when the running
//                  max grows by more than 2^8 (exact: the same stale max is
//                  used for numerator and denominator).
//    TMEM: Q at columns [0,128) (fp16 pairs), S [128,256) (one buffer: S_{j+1}
//    is issued once the softmax warps hold S_j in registers), O [256,512).
//    Epilogue: O / l * sigmoid(gate) (gemv.rs:1441-1444) written as f32.
//
//    Why 128-key tiles: a tcgen05.mma of M = 128, K = 16 costs ~68 cycles at
//    N = 64 and at N = 128 alike (N = 256: 128, the math rate), so the
//    earlier 64-key tiles ran S = Q K^T at half rate (871 -> 1,001 TFLOP/s on
//    workload 3).  Measured limit now (clock64 per phase of the issuing
//    thread): the S MMAs take ~90 cycles and the P.V MMAs ~158 in the kernel
//    (68 and 128 alone), and ~20 % of the time the issuer waits for K/V
//    chunks — shared memory (ring 176 KB + P 32 KB) and TMEM (all 512
//    columns) are both full at head dim 256 on one SM.  A CTA-pair form
//    (cta_group::2, M = 256, each CTA staging half of every K/V tile) gave
//    the same per-SM MMA times and K/V waits and was not kept.
#include <cuda_bf16.h>

#include <algorithm>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {

int encode_rows_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                     uint32_t box_inner, uint32_t box_rows, bool fp16);

namespace {

constexpr int kBM = 128;                   // query rows per CTA (UMMA M)
constexpr int kBN = 128;                   // key positions per tile (UMMA N of S = Q K^T)
constexpr int kQBox = kBM * 128;           // [128 rows x 64 dims] fp16 = 16 KB
constexpr int kSlot = 16384;               // one ring slot
constexpr int kRing = 11;                  // ring slots (176 KB)
constexpr int kVBox = 32 * 128;            // [32 keys x 64 dims] fp16 = 4 KB
constexpr int kPBox = kBM * 128;           // [128 rows x 64 keys] fp16 = 16 KB
constexpr int kPBytes = 2 * kPBox;         // P tile [128 x 128]
constexpr int kOffRing = 0;
constexpr int kOffP = kOffRing + kRing * kSlot;
constexpr int kOffRed = kOffP + kPBytes;      // row-max / row-sum exchange [2][2][128] f32
constexpr int kOffBar = kOffRed + 2 * 2 * kBM * 4;
constexpr int kPrefillSmem = kOffBar + 256 + 1024;
static_assert(kPrefillSmem <= 232448, "shared memory per CTA");
constexpr int kSoftmaxWarps = 8;              // two per TMEM lane quarter, 64 columns each
constexpr int kAttnThreads = 64 + 32 * kSoftmaxWarps;
constexpr int kTmQ = 0;    // Q as the A operand of S = Q K^T: 128 lanes x 128 columns (fp16 pairs)
constexpr int kTmS = 128;  // S, 128 columns (one buffer: S_{j+1} is issued once S_j is in registers)
constexpr int kTmO = 256;  // O accumulator, 256 columns
constexpr int kTmCols = 512;
constexpr uint32_t kIdescS = umma_idesc_f16kind(kBM, kBN, false, false, false);  // fp16 x fp16
constexpr uint32_t kIdescO = umma_idesc_f16kind(kBM, 256, false, true, false);
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct Bars {
    uint64_t full[kRing], empty[kRing];  // ring slots: TMA landed / MMAs done reading
    uint64_t q_tmem;                     // Q copied into TMEM (softmax warps)
    uint64_t s_full, s_free;             // S_j in TMEM / S_j read into registers
    uint64_t p_full, pv_done;            // P_j in shared memory / O += P_j V_j done
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

// Rows of a [128 x 256] fp16 tile held as 4 TMA boxes of [128 rows x 64]
// (128-byte swizzle) -> TMEM, column col0 + d/2 of lane `row` holding dims d
// and d+1 (the A-operand layout of tcgen05.mma); boxes [box0, box0 + nbox).
// `taddr` is the warp's lane base plus col0.
__device__ __forceinline__ void tile_rows_to_tmem(const uint8_t* tile, uint32_t taddr, int row, int box0,
                                                  int nbox) {
    for (int bi = 0; bi < nbox; bi++) {
        const int bx = box0 + bi;
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const uint4 w = *reinterpret_cast<const uint4*>(tile + bx * kQBox + sw128_off(row, c));
            v[4 * c] = __uint_as_float(w.x);
            v[4 * c + 1] = __uint_as_float(w.y);
            v[4 * c + 2] = __uint_as_float(w.z);
            v[4 * c + 3] = __uint_as_float(w.w);
        }
        tmem_st32(taddr + bx * 32, v);
    }
}

// ---------------------------------------------------------------------------
// 1. prep
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(160)
gqa_prefill_prep(const uint16_t* __restrict__ q_gate, const uint16_t* __restrict__ k_in,
                 const uint16_t* __restrict__ v_in, const float* __restrict__ q_norm,
                 const float* __restrict__ k_norm, const float* __restrict__ rope_cos,
                 const float* __restrict__ rope_sin, int T, uint16_t* __restrict__ qw,
                 uint16_t* __restrict__ kw, uint16_t* __restrict__ vw,
                 uint16_t* __restrict__ kcache, uint16_t* __restrict__ vcache, int cap, int B,
                 int* err) {
    const int g = blockIdx.x % kNumKVH;
    const int bt = blockIdx.x / kNumKVH;
    const int t = bt % T, b = bt / T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool is_q = warp < kGroup;
    const int h = g * kGroup + warp;
    const uint16_t* src = is_q ? q_gate + (((size_t)b * T + t) * kNumH + h) * 2 * kD
                               : k_in + (((size_t)b * T + t) * kNumKVH + g) * kD;
    const float* gamma = is_q ? q_norm : k_norm;
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        x[i] = bf16_bits_to_f32(src[lane + 32 * i]);
        ss = fmaf(x[i], x[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / kD) + 1e-6f);
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = x[i] * inv * (1.0f + gamma[lane + 32 * i]);
    {
        const float c = rope_cos[(size_t)t * kHalfRot + lane];
        const float s = rope_sin[(size_t)t * kHalfRot + lane];
        const float x1 = x[0], x2 = x[1];
        x[0] = x1 * c - x2 * s;
        x[1] = x2 * c + x1 * s;
    }
    if (is_q) {
        const size_t qrow = (((size_t)b * kNumH + h) * T + t) * kD;
        if (!QM_IN(qrow, kD, (size_t)B * kNumH * T * kD, err)) return;
        uint16_t* dst = qw + qrow;
#pragma unroll
        for (int i = 0; i < 8; i++) dst[lane + 32 * i] = f16_bits_rn(x[i] * 0.0625f);
    } else {
        const size_t row = (((size_t)b * kNumKVH + g) * cap + t) * kD;
        const size_t wrow = (((size_t)b * kNumKVH + g) * T + t) * kD;
        if (!QM_IN(row, kD, (size_t)B * kNumKVH * cap * kD, err) ||
            !QM_IN(wrow, kD, (size_t)B * kNumKVH * T * kD, err))
            return;
        const uint16_t* vs = v_in + (((size_t)b * T + t) * kNumKVH + g) * kD;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = lane + 32 * i;
            const uint16_t vb = vs[e];
            kcache[row + e] = bf16_bits_rn(x[i]);
            vcache[row + e] = vb;
            kw[wrow + e] = f16_bits_rn(x[i]);
            vw[wrow + e] = __half_as_ushort(__float2half_rn(fminf(fmaxf(bf16_bits_to_f32(vb), -65504.f), 65504.f)));
        }
    }
}

// ---------------------------------------------------------------------------
// 2. flash attention
// ---------------------------------------------------------------------------
// Shared memory holds a ring of 16 KB slots that the TMA producer fills in
// the order the consumers take them: the Q tile (4 slots, copied into TMEM by
// the softmax warps and released), then K_0, and for each tile j: K_{j+1}
// (4 slots of [128 keys x 64 dims]) and V_j (4 slots of [32 keys x 256 dims],
// each as 4 boxes of [32 x 64]) — the issue order S_0, S_1, PV_0, S_2, PV_1,
// ...  Slot n of the sequence is slot n % kRing, phase (n / kRing) & 1.
__global__ void __launch_bounds__(kAttnThreads, 1)
gqa_prefill_attn(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                 const __grid_constant__ CUtensorMap tmv, const uint16_t* __restrict__ q_gate,
                 float* __restrict__ out, int T, int nqt, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t ring = sbase + kOffRing;

    // heaviest query tiles first; the 16 heads of one tile are adjacent so the
    // 4 heads of a KV group read the same K/V tiles from L2
    const int h = blockIdx.x % kNumH;
    const int qt = nqt - 1 - (int)(blockIdx.x / kNumH);
    const int b = blockIdx.y;
    const int g = h / kGroup;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = qt * kBM;
    const int n_tiles = min(qt + 1, (T + kBN - 1) / kBN);  // kBM == kBN: tile qt holds the diagonal

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRing; i++) {
            mbar_init(smem_u32(&bars->full[i]), 1);
            mbar_init(smem_u32(&bars->empty[i]), 1);
        }
        mbar_init(smem_u32(&bars->q_tmem), kSoftmaxWarps);
        mbar_init(smem_u32(&bars->s_full), 1);
        mbar_init(smem_u32(&bars->s_free), kSoftmaxWarps);
        mbar_init(smem_u32(&bars->p_full), kSoftmaxWarps);
        mbar_init(smem_u32(&bars->pv_done), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            prefetch_tmap(&tmq);
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
            const int zc = b * kNumKVH + g;
            int n = 0;
            bool ok = true;
            // slot of chunk n, once the chunk kRing places earlier has been released
            auto claim = [&](int& slot) -> bool {
                slot = n % kRing;
                if (n >= kRing && !mbar_wait_bounded(smem_u32(&bars->empty[slot]), ((n / kRing) - 1) & 1,
                                                     abort_flag, err))
                    return false;
                mbar_arrive_expect_tx(smem_u32(&bars->full[slot]), kSlot);
                return true;
            };
            for (int sub = 0; sub < 4; sub++) {  // Q: chunks 0..3 (slots 0..3, contiguous)
                int slot;
                claim(slot);
                if (QM_IN(slot * kSlot, kSlot, kRing * kSlot, err))
                    tma_load_3d(ring + slot * kSlot, &tmq, sub * 64, q0, b * kNumH + h,
                                smem_u32(&bars->full[slot]));
                n++;
            }
            auto load_k = [&](int j) {
                for (int c = 0; c < 4 && ok; c++) {
                    int slot;
                    if (!(ok = claim(slot))) break;
                    if (QM_IN(slot * kSlot, kSlot, kRing * kSlot, err))
                        tma_load_3d(ring + slot * kSlot, &tmk, c * 64, j * kBN, zc, smem_u32(&bars->full[slot]));
                    n++;
                }
            };
            auto load_v = [&](int j) {
                for (int c = 0; c < 4 && ok; c++) {
                    int slot;
                    if (!(ok = claim(slot))) break;
                    for (int d = 0; d < 4; d++)
                        if (QM_IN(slot * kSlot + d * kVBox, kVBox, kRing * kSlot, err))
                            tma_load_3d(ring + slot * kSlot + d * kVBox, &tmv, d * 64, j * kBN + c * 32, zc,
                                        smem_u32(&bars->full[slot]));
                    n++;
                }
            };
            load_k(0);
            for (int j = 0; j < n_tiles && ok; j++) {
                if (j + 1 < n_tiles) load_k(j + 1);
                load_v(j);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ----------------------------
        if (lane == 0) {
            int n = 4;  // chunks 0..3 held Q
            // Q reaches TMEM through the softmax warps (q_tmem); its slots are then free
            bool ok = mbar_wait_bounded(smem_u32(&bars->q_tmem), 0, abort_flag, err);
            if (ok)
                for (int i = 0; i < 4; i++) mbar_arrive(smem_u32(&bars->empty[i]));
            auto take = [&](int& slot) -> bool {
                slot = n % kRing;
                if (!mbar_wait_bounded(smem_u32(&bars->full[slot]), (n / kRing) & 1, abort_flag, err))
                    return false;
                tc_fence_after();
                return true;
            };
            // S_j = Q K_j^T: 16 MMAs (K = 16 dims each), A = Q from TMEM
            auto issue_s = [&]() -> bool {
                for (int c = 0; c < 4; c++) {
                    int slot;
                    if (!take(slot)) return false;
#pragma unroll
                    for (int k4 = 0; k4 < 4; k4++) {
                        const int kk = c * 4 + k4;
                        const uint64_t bd = umma_sdesc(ring + slot * kSlot + k4 * 32, 16, 1024);
                        umma_f16_ts(tm + kTmS, tm + kTmQ + kk * 8, bd, kIdescS, kk > 0 ? 1u : 0u);
                    }
                    umma_commit(smem_u32(&bars->empty[slot]));
                    n++;
                }
                umma_commit(smem_u32(&bars->s_full));
                return true;
            };
            // O += P_j V_j: 8 MMAs (K = 16 keys each), P from shared memory,
            // V read MN-major from its [key][dim] boxes
            auto issue_pv = [&](int j) -> bool {
                if (!mbar_wait_bounded(smem_u32(&bars->p_full), j & 1, abort_flag, err)) return false;
                tc_fence_after();
                const uint32_t pbase = sbase + kOffP;
                for (int c = 0; c < 4; c++) {
                    int slot;
                    if (!take(slot)) return false;
#pragma unroll
                    for (int k2 = 0; k2 < 2; k2++) {
                        const int kk = c * 2 + k2;
                        const uint64_t ad = umma_sdesc(pbase + (kk >> 2) * kPBox + (kk & 3) * 32, 16, 1024);
                        const uint64_t bd = umma_sdesc(ring + slot * kSlot + k2 * 2048, kVBox, 1024);
                        umma_bf16_ss(tm + kTmO, ad, bd, kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(smem_u32(&bars->empty[slot]));
                    n++;
                }
                umma_commit(smem_u32(&bars->pv_done));
                return true;
            };
            if (ok) ok = issue_s();
            for (int j = 0; ok && j < n_tiles; j++) {
                if (j + 1 < n_tiles) {
                    // S_{j+1} overwrites S_j: wait until the softmax warps hold S_j in registers
                    ok = mbar_wait_bounded(smem_u32(&bars->s_free), j & 1, abort_flag, err);
                    if (ok) ok = issue_s();
                }
                if (ok) ok = issue_pv(j);
            }
        }
    } else {
        // ------------------------------ softmax (warps 2..9) -----------------
        // Two warps per TMEM lane quarter: warp w reads lanes 32*(w%4).. and
        // half (w-2)/4 of the 128 score columns.  The row max is exchanged
        // through shared memory (parity double buffer, one named barrier of
        // the quarter's 64 threads per tile); row sums stay per half until
        // the epilogue.  Both halves see the same row max, so they take the
        // same rescale decisions.
        const int quarter = warp & 3;             // TMEM lanes 32*quarter .. +31
        const int half = (warp - 2) >> 2;         // score columns [64*half, 64*half+64)
        const int r = quarter * 32 + lane;        // query row within the tile
        const int qp = q0 + r;                    // query position
        const int bar_id = 1 + quarter;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        float* red = reinterpret_cast<float*>(smem + kOffRed);  // [parity][half][row]
        float m_used = -INFINITY, l = 0.f;
        // Q tile (ring slots 0..3) -> TMEM, this warp's rows and dims
        // [128 half, 128 half + 128), once: the S MMAs read it from there
        bool ok = mbar_wait_bounded(smem_u32(&bars->full[2 * half]), 0, abort_flag, err);
        ok = ok && mbar_wait_bounded(smem_u32(&bars->full[2 * half + 1]), 0, abort_flag, err);
        if (ok) {
            tile_rows_to_tmem(smem + kOffRing, tm + lane_addr + kTmQ, r, 2 * half, 2);
            tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars->q_tmem));
        for (int j = 0; j < n_tiles; j++) {
            ok = ok && mbar_wait_bounded(smem_u32(&bars->s_full), j & 1, abort_flag, err);
            float s[64];
            if (ok) {
                tc_fence_after();
                tmem_ld32(tm + lane_addr + kTmS + half * 64, s);
                tmem_ld32(tm + lane_addr + kTmS + half * 64 + 32, s + 32);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int c = 0; c < 64; c++) s[c] = 0.f;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars->s_free));
            // causal + length mask (only tiles that reach the diagonal or T)
            const int kp0 = j * kBN + half * 64;
            if (kp0 + 63 > q0 || kp0 + 64 > T) {
                const int lim = min(qp, T - 1) - kp0;  // columns c <= lim are visible
#pragma unroll
                for (int c = 0; c < 64; c++)
                    if (c > lim) s[c] = -INFINITY;
            }
            float m4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) m4[i] = fmaxf(s[i], s[i + 4]);
#pragma unroll
            for (int c = 8; c < 64; c += 4) {
#pragma unroll
                for (int i = 0; i < 4; i++) m4[i] = fmaxf(m4[i], s[c + i]);
            }
            float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            const int par = j & 1;
            if (QM_IN((par * 2 + half) * kBM + r, 1, 2 * 2 * kBM, err)) red[(par * 2 + half) * kBM + r] = mx;
            named_bar_sync(bar_id, 64);
            mx = fmaxf(mx, red[(par * 2 + (half ^ 1)) * kBM + r]);
            const float m_new = fmaxf(m_used, mx * kLog2e);
            bool rescale = false;
            float factor = 1.f;
            if (m_used == -INFINITY) {
                m_used = m_new;
            } else if (m_new > m_used + kRescaleThreshold) {
                factor = ex2_approx(m_used - m_new);
                m_used = m_new;
                rescale = true;
            }
            l *= factor;
            const float nm = -m_used;
            uint32_t pk[32];
            float r4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
                const float p0 = ex2_approx(fmaf(s[c], kLog2e, nm));
                const float p1 = ex2_approx(fmaf(s[c + 1], kLog2e, nm));
                r4[(c >> 1) & 3] += p0 + p1;
                pk[c / 2] = pack_f16x2_rn(p0, p1);
            }
            l += (r4[0] + r4[1]) + (r4[2] + r4[3]);
            // PV_{j-1} must be complete: it read the P buffer, and O is
            // stable for rescaling.
            if (j >= 1)
                ok = ok && mbar_wait_bounded(smem_u32(&bars->pv_done), (j - 1) & 1, abort_flag, err);
            if (ok) {
                tc_fence_after();
                if (__any_sync(0xffffffffu, rescale) && j >= 1) {
#pragma unroll 1
                    for (int c = 0; c < 4; c++) {
                        float o[32];
                        const uint32_t oa = tm + lane_addr + kTmO + half * 128 + c * 32;
                        tmem_ld32(oa, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] *= factor;
                        tmem_st32(oa, o);
                    }
                    tmem_st_wait();
                }
                // this half's 64 keys = one 128-byte row of P box `half`
                uint8_t* pbox = smem + kOffP + half * kPBox;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    uint4 v = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                    if (QM_IN(half * kPBox + sw128_off(r, c), 16, kPBytes, err))
                        *reinterpret_cast<uint4*>(pbox + sw128_off(r, c)) = v;
                }
                fence_proxy_async_shared();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars->p_full));
        }
        // ------------------------------ epilogue ------------------------------
        // the two halves' row sums (the exchange buffer of the next parity is
        // free: its last readers passed this quarter's barrier of the last tile)
        const int pe = n_tiles & 1;
        if (QM_IN((pe * 2 + half) * kBM + r, 1, 2 * 2 * kBM, err)) red[(pe * 2 + half) * kBM + r] = l;
        named_bar_sync(bar_id, 64);
        l += red[(pe * 2 + (half ^ 1)) * kBM + r];
        const int jl = n_tiles - 1;
        ok = ok && mbar_wait_bounded(smem_u32(&bars->pv_done), jl & 1, abort_flag, err);
        if (ok) {
            tc_fence_after();
            const float inv_l = 1.0f / l;
            const size_t orow_off = (((size_t)b * T + (qp < T ? qp : 0)) * kNumH + h) * kD + half * 128;
            const bool valid = qp < T && QM_IN(orow_off, 128, (size_t)gridDim.y * T * kNumH * kD, err);
            const uint16_t* grow = q_gate + (((size_t)b * T + (valid ? qp : 0)) * kNumH + h) * 2 * kD + kD
                                   + half * 128;
            float* orow = out + (((size_t)b * T + (valid ? qp : 0)) * kNumH + h) * kD + half * 128;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float o[32];
                tmem_ld32(tm + lane_addr + kTmO + half * 128 + c * 32, o);
                tmem_ld_wait();
                if (valid) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        const uint2 gb = *reinterpret_cast<const uint2*>(grow + c * 32 + i);
                        float4 w;
                        w.x = o[i + 0] * inv_l * (1.0f / (1.0f + __expf(-bf16_bits_to_f32(gb.x & 0xffffu))));
                        w.y = o[i + 1] * inv_l * (1.0f / (1.0f + __expf(-bf16_bits_to_f32(gb.x >> 16))));
                        w.z = o[i + 2] * inv_l * (1.0f / (1.0f + __expf(-bf16_bits_to_f32(gb.y & 0xffffu))));
                        w.w = o[i + 3] * inv_l * (1.0f / (1.0f + __expf(-bf16_bits_to_f32(gb.y >> 16))));
                        *reinterpret_cast<float4*>(orow + c * 32 + i) = w;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, kTmCols);
    }
}

}  // namespace

// fp16 q [B,16,T,256], k and v [B,4,T,256]
size_t gqa_prefill_ws_bytes(int batch, int T) {
    return (size_t)batch * (kNumH + 2 * kNumKVH) * T * kD * 2;
}

cudaError_t launch_gqa_prefill(qm_ctx* ctx, const qm_gqa_params* prm, qm_kv* kv, int T,
                               const uint16_t* q_gate, const uint16_t* k, const uint16_t* v,
                               float* out) {
    const int B = kv->batch;
    cudaStream_t st = ctx->stream;
    uint16_t* qw = static_cast<uint16_t*>(ctx->ws);
    uint16_t* kw = qw + (size_t)B * kNumH * T * kD;
    uint16_t* vw = kw + (size_t)B * kNumKVH * T * kD;
    {
        TimedLaunch tl(ctx, "gqa_prefill_prep");
        gqa_prefill_prep<<<(unsigned)((size_t)B * T * kNumKVH), 160, 0, st>>>(
            q_gate, k, v, prm->q_norm, prm->k_norm, prm->rope_cos, prm->rope_sin, T, qw, kw, vw,
            kv->k, kv->v, kv->capacity, B, ctx->d_err);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    CUtensorMap tmq, tmk, tmv;
    if (encode_rows_tmap(&tmq, qw, kD, (uint64_t)T, (uint64_t)B * kNumH, 64, kBM, true) != QM_OK ||
        encode_rows_tmap(&tmk, kw, kD, (uint64_t)T, (uint64_t)B * kNumKVH, 64, kBN, true) != QM_OK ||
        encode_rows_tmap(&tmv, vw, kD, (uint64_t)T, (uint64_t)B * kNumKVH, 64, 32, true) != QM_OK)
        return cudaErrorInvalidValue;
    static std::atomic<uint64_t> attr_set{0};
    e = set_smem_once(attr_set, ctx->device, gqa_prefill_attn, kPrefillSmem);
    if (e != cudaSuccess) return e;
    const int nqt = (T + kBM - 1) / kBM;
    dim3 grid(nqt * kNumH, B);
    {
        TimedLaunch tl(ctx, "gqa_prefill_attn");
        gqa_prefill_attn<<<grid, kAttnThreads, kPrefillSmem, st>>>(tmq, tmk, tmv, q_gate, out, T, nqt,
                                                          ctx->d_err);
    }
    e = cudaGetLastError();
    if (e == cudaSuccess) ctx->launches += 1;
    return e;
}

}  // namespace qm

using namespace qm;

extern "C" int qm_gqa_prefill(qm_ctx* c, const qm_gqa_params* p, qm_kv* kv, int T,
                              const uint16_t* q_gate, const uint16_t* k, const uint16_t* v,
                              float* out) {
    if (!c) return QM_E_ARG;
    if (!p || !p->q_norm || !p->k_norm || !p->rope_cos || !p->rope_sin || p->max_pos <= 0)
        return set_error(c, QM_E_ARG, "GQA params: null pointer or max_pos <= 0");
    if (!kv || !q_gate || !k || !v || !out || T <= 0)
        return set_error(c, QM_E_ARG, "qm_gqa_prefill: null pointer or T <= 0");
    if (kv->ctx != c) return set_error(c, QM_E_MISMATCH, "cache belongs to another context");
    if (kv->nkv != kNumKVH)
        return set_error(c, QM_E_UNSUPPORTED, "qm_gqa_prefill: head-sharded caches are decode-only");
    if (T > kv->capacity) return set_error(c, QM_E_RANGE, "qm_gqa_prefill: T exceeds the cache capacity");
    if (T > p->max_pos) return set_error(c, QM_E_RANGE, "qm_gqa_prefill: T exceeds the RoPE table");
    if (((uintptr_t)out & 15) || ((uintptr_t)q_gate & 15))
        return set_error(c, QM_E_ARG, "qm_gqa_prefill: out and q_gate must be 16-byte aligned");
    cudaSetDevice(c->device);
    int rc = ensure_workspace(c, gqa_prefill_ws_bytes(kv->batch, T));
    if (rc) return rc;
    cudaError_t e = launch_gqa_prefill(c, p, kv, T, q_gate, k, v, out);
    if (e != cudaSuccess) return cuda_error(c, e, "gqa_prefill launch");
    kv->seq_len = T;
    return QM_OK;
}
