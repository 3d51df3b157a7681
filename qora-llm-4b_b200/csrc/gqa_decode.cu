// GQA decode: one new token for B sequences against a bf16 KV cache.
//
// Replaces src/gemv.rs:927-1011 (CPU, rayon over 16 heads) and
// src/gpu_inference.rs:269-349 (wgpu: re-concatenates the cache and repeats
// every KV head 4x each token).  Three launches:
//
//  1. prep     (B*4 CTAs)  QK-RMSNorm(1+g) + partial RoPE of the new q/k,
//               bf16 append of k/v at position L, q split into bf16 hi+lo.
//  2. attn     (nsplit x 4 x B CTAs)  split-KV attention over the L cached
//               positions.  A producer warp streams 64-position K/V tiles
//               with TMA (128-byte swizzle) into a 3-stage mbarrier ring;
//               4 consumer warps run q.K^T and P.V on the tensor cores.
//               The 4 query heads of a KV group share every K/V tile; q and
//               P enter the MMA as bf16 hi+lo pairs so the products keep
//               ~16 mantissa bits (the reference is f32 throughout).
//  3. combine  (B*16 CTAs)  log-sum-exp merge of the split partials plus the
//               new token itself in f32, then the sigmoid gate.
//
// The cache stays in place: the reference's per-token Tensor::cat (O(L) copy)
// becomes one 1 KB write per (sequence, KV head).
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {
namespace {

constexpr int kTile = 64;                       // positions per K/V tile
constexpr int kStages = 3;
constexpr int kSubBytes = 64 * 128;             // one 64x64 bf16 box (128 B rows)
constexpr int kTileBytes = 4 * kSubBytes;       // 64 positions x 256 dims
constexpr int kStageBytes = 2 * kTileBytes;     // K + V
constexpr int kAttnSmem = kStages * kStageBytes + 1024 /*align*/ + 128 /*barriers*/;
constexpr float kLog2e = 1.4426950408889634f;

struct Plan {
    int ntiles = 0, nsplit = 0, tps = 0;
};

// B * nkv (sequence, KV head) pairs share the SMs.
Plan plan_for(int B, int nkv, int64_t L, int num_sms) {
    Plan p;
    p.ntiles = (int)((L + kTile - 1) / kTile);
    if (p.ntiles == 0) return p;
    const int64_t units = (int64_t)B * nkv;
    const int64_t total = (int64_t)p.ntiles * units;
    const int64_t waves = std::max<int64_t>(1, total / ((int64_t)num_sms * 8));
    const int64_t target = waves * num_sms;
    int ns = (int)std::min<int64_t>(p.ntiles, std::max<int64_t>(1, (target + units - 1) / units));
    p.tps = (p.ntiles + ns - 1) / ns;
    p.nsplit = (p.ntiles + p.tps - 1) / p.tps;
    return p;
}

struct WsLayout {
    size_t q_bf, q_f32, kn, part_o, part_ml, total;
};

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace for B sequences x nkv KV heads (nkv * 4 query heads).
WsLayout ws_layout(int B, int nkv, int nsplit) {
    WsLayout w;
    const size_t nh = (size_t)nkv * kGroup;
    size_t off = 0;
    w.q_bf = off;    off += al256((size_t)B * nh * 2 * kD * 2);
    w.q_f32 = off;   off += al256((size_t)B * nh * kD * 4);
    w.kn = off;      off += al256((size_t)B * nkv * kD * 4);
    w.part_o = off;  off += al256((size_t)B * nh * std::max(nsplit, 1) * kD * 4);
    w.part_ml = off; off += al256((size_t)B * nh * std::max(nsplit, 1) * 2 * 4);
    w.total = off;
    return w;
}

// ---------------------------------------------------------------------------
// 1. prep: gemv.rs:945-955 for the new token
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(160)
gqa_prep_kernel(const float* __restrict__ q_gate, const float* __restrict__ k_new,
                const float* __restrict__ v_new, const float* __restrict__ q_norm,
                const float* __restrict__ k_norm, const float* __restrict__ rope_cos,
                const float* __restrict__ rope_sin, int64_t pos, uint16_t* __restrict__ kcache,
                uint16_t* __restrict__ vcache, int cap, uint16_t* __restrict__ q_bf,
                float* __restrict__ q_f32, float* __restrict__ kn_out, int kv_lo, int nkv, int b0) {
    // the attention kernel may start now: its K/V loads read only positions the
    // preceding calls have finished writing, and it waits before reading q
    pdl_launch_dependents();
    pdl_wait();  // the inputs may come from the preceding kernel
    // gl: KV head within the cache's range; g, h: model KV / query head (inputs)
    const int b = b0 + blockIdx.x / nkv, gl = blockIdx.x % nkv, g = kv_lo + gl;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool is_q = warp < kGroup;
    const int h = g * kGroup + warp;
    const size_t hl = ((size_t)b * nkv + gl) * kGroup + warp;  // local query-head row
    const float* src = is_q ? q_gate + ((size_t)b * kNumH + h) * 2 * kD
                            : k_new + ((size_t)b * kNumKVH + g) * kD;
    const float* gamma = is_q ? q_norm : k_norm;
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        x[i] = src[lane + 32 * i];
        ss = fmaf(x[i], x[i], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / kD) + 1e-6f);  // gemv.rs:591
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = x[i] * inv * (1.0f + gamma[lane + 32 * i]);
    // split-half partial RoPE (gemv.rs:604-627): pair (lane, lane + 32)
    {
        const float c = rope_cos[pos * kHalfRot + lane];
        const float s = rope_sin[pos * kHalfRot + lane];
        const float x1 = x[0], x2 = x[1];
        x[0] = x1 * c - x2 * s;
        x[1] = x2 * c + x1 * s;
    }
    if (is_q) {
        uint16_t* qh = q_bf + hl * 2 * kD;
        float* qf = q_f32 + hl * kD;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = lane + 32 * i;
            const float qs = x[i] * 0.0625f;  // scale 1/sqrt(256) (gemv.rs:959), exact
            const uint16_t hi = bf16_bits_rn(qs);
            const uint16_t lo = bf16_bits_rn(qs - bf16_bits_to_f32(hi));
            qf[e] = qs;
            qh[e] = hi;
            qh[kD + e] = lo;
        }
    } else {
        const size_t row = (((size_t)b * nkv + gl) * cap + pos) * kD;
        const float* vs = v_new + ((size_t)b * kNumKVH + g) * kD;
        float* kn = kn_out + ((size_t)b * nkv + gl) * kD;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int e = lane + 32 * i;
            kn[e] = x[i];
            kcache[row + e] = bf16_bits_rn(x[i]);
            vcache[row + e] = bf16_bits_rn(vs[e]);
        }
    }
}

// ---------------------------------------------------------------------------
// 2. split-KV attention over cached positions [0, L)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t swz_addr(uint32_t base, int pos, int dim) {
    // 4 boxes of [64 positions x 64 dims]; within a box row = 128 B and the
    // 16-byte chunk index is XOR-ed with (row % 8) (TMA SWIZZLE_128B).
    return base + (uint32_t)((dim >> 6) * kSubBytes + pos * 128 +
                             ((((dim & 63) >> 3) ^ (pos & 7)) << 4));
}

// Consumer side of the split-KV attention over tiles [tile0, tile0 + ntiles)
// (positions below pos_end count): warp w (0..3) owns positions [16w, 16w+16)
// of each 64-position tile of the stage ring; qa holds the 4 query heads' q
// as bf16 A fragments, hi parts in rows 0-3 and lo parts in rows 4-7.  o, m_run
// and l_run are the warp's running (unnormalised) output, maximum and sum.
__device__ __forceinline__ void attend_tiles(uint32_t sbase, uint64_t* full, uint64_t* empty,
                                             volatile int* abort_flag, int* err, const uint32_t (&qa)[16][2],
                                             int tile0, int ntiles, int pos_end, int warp, int lane,
                                             float (&o)[32][2], float& m_run, float& l_run) {
    const int quad = lane & 3;
    for (int it = 0; it < ntiles; it++) {
        const int st = it % kStages, round = it / kStages;
        const bool ok = mbar_wait_bounded(smem_u32(&full[st]), round & 1, abort_flag, err);
        if (ok) {
            const uint32_t kb = sbase + st * kStageBytes;
            const uint32_t vb = kb + kTileBytes;
            // ---- S = q . K^T for 16 positions (2 n-tiles of 8) ----
            float c[2][2];
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                c[nt][0] = c[nt][1] = 0.f;
                const int pos = warp * 16 + nt * 8 + (lane & 7);
#pragma unroll
                for (int k2 = 0; k2 < 8; k2++) {
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4(swz_addr(kb, pos, k2 * 32 + (lane >> 3) * 8), r0, r1, r2, r3);
                    mma_bf16_top(c[nt][0], c[nt][1], qa[2 * k2][0], qa[2 * k2][1], r0, r1);
                    mma_bf16_top(c[nt][0], c[nt][1], qa[2 * k2 + 1][0], qa[2 * k2 + 1][1], r2, r3);
                }
            }
            // ---- online softmax; hi and lo rows sit 16 lanes apart ----
            const int pbase = (tile0 + it) * kTile + warp * 16 + quad * 2;
            float s[2][2];
            float tmax = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float v = c[nt][j] + __shfl_xor_sync(0xffffffffu, c[nt][j], 16);
                    if (pbase + nt * 8 + j >= pos_end) v = -INFINITY;
                    s[nt][j] = v;
                    tmax = fmaxf(tmax, v);
                }
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
            const float m_new = fmaxf(m_run, tmax);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float corr = exp2f((m_run - m_use) * kLog2e);
            float p[2][2], rs = 0.f;
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    p[nt][j] = exp2f((s[nt][j] - m_use) * kLog2e);
                    rs += p[nt][j];
                }
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            l_run = l_run * corr + rs;
            m_run = m_new;
            if (__any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll
                for (int n = 0; n < 32; n++) {
                    o[n][0] *= corr;
                    o[n][1] *= corr;
                }
            }
            // P as bf16 hi (rows 0-3, lanes 0-15) + lo (rows 4-7, lanes 16-31)
            uint16_t pb[2][2];
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint16_t hi = bf16_bits_rn(p[nt][j]);
                    pb[nt][j] = (lane < 16) ? hi : bf16_bits_rn(p[nt][j] - bf16_bits_to_f32(hi));
                }
            const uint32_t a0 = pack_bf16(pb[0][0], pb[0][1]);
            const uint32_t a2 = pack_bf16(pb[1][0], pb[1][1]);
            // ---- rows at or past the end of the range: P is 0 there, but cache
            // memory beyond seq_len may hold anything (a caller's buffer) and
            // 0 * NaN would poison O, so this warp's V rows there become zeros ----
            const int wpos0 = (tile0 + it) * kTile + warp * 16;
            if (wpos0 + 16 > pos_end) {
                for (int e = lane; e < 16 * 32; e += 32) {
                    const int i = e >> 5, c = e & 31;
                    if (wpos0 + i >= pos_end)
                        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                                         swz_addr(vb, warp * 16 + i, c * 8)),
                                     "r"(0u)
                                     : "memory");
                }
                __syncwarp();
                fence_proxy_async_shared();  // before TMA refills this stage
            }
            // ---- O += P . V over 256 dims ----
            const int mi = lane >> 3;
            const int vpos = warp * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
            for (int dn = 0; dn < 16; dn++) {
                uint32_t r0, r1, r2, r3;
                ldsm_x4_t(swz_addr(vb, vpos, dn * 16 + (mi >> 1) * 8), r0, r1, r2, r3);
                mma_bf16_top(o[2 * dn][0], o[2 * dn][1], a0, a2, r0, r1);
                mma_bf16_top(o[2 * dn + 1][0], o[2 * dn + 1][1], a0, a2, r2, r3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[st]));
    }

}

// The same attention with the operands swapped, as the fused kernel runs it:
// per warp and tile, S^T [16 positions x 8] = K [16 x 256] . Q^T, where the 8
// columns are the 4 heads' q in bf16 hi (columns 0-3) and lo (4-7), so every
// row of the 16-row MMA is a position (16 MMAs a tile instead of 32), and
// O^T [256 dims x 8] += V^T [256 x 16 positions] . P^T (16 instead of 32).
// Lane l holds scores of heads 2(q & 1) + j, j = 0, 1 (q = l & 3) at
// positions l/4 and l/4 + 8 of its warp's 16, and its O^T accumulator columns
// 2q, 2q+1 are the hi or lo parts of the same two heads, so the online
// softmax rescales them in place.  P^T enters the MMA as the B operand: lane
// l needs P at positions 2q, 2q+1, 2q+8, 2q+9 for column l/4, which 8
// shuffles collect.  qb are the q B fragments (the same registers as the A
// fragments of attend_tiles); oc[mt] holds dims 16mt + l/4 (c0, c1) and
// 16mt + l/4 + 8 (c2, c3), columns 2q, 2q+1.
__device__ __forceinline__ void attend_tiles_t(uint32_t sbase, uint64_t* full, uint64_t* empty,
                                               volatile int* abort_flag, int* err, const uint32_t (&qb)[16][2],
                                               int tile0, int ntiles, int pos_end, int warp, int lane,
                                               float (&oc)[16][4], float (&m_run)[2], float (&l_run)[2]) {
    const int quad = lane & 3, g8 = lane >> 2;
    const int hsel = g8 & 3, hl = g8 >> 2;          // B column of this lane: head, hi (0) / lo (1)
    const int src_a = (2 * quad) * 4 + (hsel >> 1);  // holder of positions 2q and 2q + 8
    const int src_b = src_a + 4;                     // holder of positions 2q + 1 and 2q + 9
    const int krow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // ldmatrix rows (K, A operand)
    const int kdim = (lane >> 4) * 8;
    const int vrow = warp * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;  // ldmatrix.trans rows (V^T)
    const int vdim = ((lane >> 3) & 1) * 8;
    for (int it = 0; it < ntiles; it++) {
        const int st = it % kStages, round = it / kStages;
        const bool ok = mbar_wait_bounded(smem_u32(&full[st]), round & 1, abort_flag, err);
        if (ok) {
            const uint32_t kb = sbase + st * kStageBytes;
            const uint32_t vb = kb + kTileBytes;
            // four independent accumulation chains over the 256 dims (a quarter of
            // the dependent MMA latency), summed in a fixed order
            float cq[4][4];
#pragma unroll
            for (int a = 0; a < 4; a++) cq[a][0] = cq[a][1] = cq[a][2] = cq[a][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 16; kk++) {
                uint32_t r0, r1, r2, r3;
                ldsm_x4(swz_addr(kb, krow, kk * 16 + kdim), r0, r1, r2, r3);
                mma_bf16_16816(cq[kk & 3], r0, r1, r2, r3, qb[kk][0], qb[kk][1]);
            }
            float c[4];
#pragma unroll
            for (int i = 0; i < 4; i++) c[i] = (cq[0][i] + cq[1][i]) + (cq[2][i] + cq[3][i]);
            // hi + lo columns (lanes q and q ^ 2); s[j][i]: head 2(q&1)+j, position g8 + 8i
            float s[2][2];
            s[0][0] = c[0] + __shfl_xor_sync(0xffffffffu, c[0], 2);
            s[1][0] = c[1] + __shfl_xor_sync(0xffffffffu, c[1], 2);
            s[0][1] = c[2] + __shfl_xor_sync(0xffffffffu, c[2], 2);
            s[1][1] = c[3] + __shfl_xor_sync(0xffffffffu, c[3], 2);
            const int p0 = (tile0 + it) * kTile + warp * 16 + g8;
#pragma unroll
            for (int i = 0; i < 2; i++)
                if (p0 + 8 * i >= pos_end) s[0][i] = s[1][i] = -INFINITY;
            // Lazy rescaling: P is taken against the warp's reference maximum
            // m_run, which moves (a reduction over the warp, then O and the sums
            // rescaled) only when some score exceeds it by more than 2^8 in
            // exp2 units; otherwise a tile costs no cross-lane reduction.  The
            // sums stay per lane until the end (the result does not depend on
            // the reference: numerator and denominator use the same one).
            bool grow = false;
#pragma unroll
            for (int j = 0; j < 2; j++)
                grow |= (fmaxf(s[j][0], s[j][1]) - m_run[j]) * kLog2e > 8.0f;  // -inf - -inf: NaN, false
            if (__any_sync(0xffffffffu, grow)) {
                float corr[2];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float tmax = fmaxf(s[j][0], s[j][1]);
                    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
                    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
                    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
                    const float m_new = fmaxf(m_run[j], tmax);
                    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
                    corr[j] = exp2f((m_run[j] - m_use) * kLog2e);  // m_run -inf: 0 (nothing to keep)
                    l_run[j] *= corr[j];
                    m_run[j] = m_new;
                }
#pragma unroll
                for (int mt = 0; mt < 16; mt++) {
                    oc[mt][0] *= corr[0];
                    oc[mt][1] *= corr[1];
                    oc[mt][2] *= corr[0];
                    oc[mt][3] *= corr[1];
                }
            }
            float p[2][2];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float m_use = (m_run[j] == -INFINITY) ? 0.f : m_run[j];
                p[j][0] = exp2f((s[j][0] - m_use) * kLog2e);
                p[j][1] = exp2f((s[j][1] - m_use) * kLog2e);
                l_run[j] += p[j][0] + p[j][1];
            }
            // P^T fragment: column (hsel, hl) at positions 2q, 2q+1 (b0) and 2q+8, 2q+9 (b1)
            const float a00 = __shfl_sync(0xffffffffu, p[0][0], src_a), a10 = __shfl_sync(0xffffffffu, p[1][0], src_a);
            const float a01 = __shfl_sync(0xffffffffu, p[0][1], src_a), a11 = __shfl_sync(0xffffffffu, p[1][1], src_a);
            const float b00 = __shfl_sync(0xffffffffu, p[0][0], src_b), b10 = __shfl_sync(0xffffffffu, p[1][0], src_b);
            const float b01 = __shfl_sync(0xffffffffu, p[0][1], src_b), b11 = __shfl_sync(0xffffffffu, p[1][1], src_b);
            const bool odd = hsel & 1;
            const float pv[4] = {odd ? a10 : a00, odd ? b10 : b00, odd ? a11 : a01, odd ? b11 : b01};
            uint16_t pb[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint16_t hi = bf16_bits_rn(pv[k]);
                pb[k] = hl ? bf16_bits_rn(pv[k] - bf16_bits_to_f32(hi)) : hi;
            }
            const uint32_t pb0 = pack_bf16(pb[0], pb[1]), pb1 = pack_bf16(pb[2], pb[3]);
            // rows at or past the end of the range: P is 0 there, but the cache may
            // hold anything (NaN) and 0 * NaN would poison O, so those V rows become 0
            const int wpos0 = (tile0 + it) * kTile + warp * 16;
            if (wpos0 + 16 > pos_end) {
                for (int e = lane; e < 16 * 32; e += 32) {
                    const int i = e >> 5, cc = e & 31;
                    if (wpos0 + i >= pos_end)
                        asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                                         swz_addr(vb, warp * 16 + i, cc * 8)),
                                     "r"(0u)
                                     : "memory");
                }
                __syncwarp();
                fence_proxy_async_shared();  // before TMA refills this stage
            }
#pragma unroll
            for (int mt = 0; mt < 16; mt++) {
                uint32_t r0, r1, r2, r3;
                ldsm_x4_t(swz_addr(vb, vrow, mt * 16 + vdim), r0, r1, r2, r3);
                mma_bf16_16816(oc[mt], r0, r1, r2, r3, pb0, pb1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[st]));
    }
    // the warp's sums over its 16 positions (lanes with the same heads)
#pragma unroll
    for (int j = 0; j < 2; j++) {
        l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 4);
        l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 8);
        l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 16);
    }
}

__global__ void __launch_bounds__(160, 1)
gqa_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                const uint16_t* __restrict__ q_bf, float* __restrict__ part_o,
                float* __restrict__ part_ml, int L, int tps, int nsplit, int nkv, int b0, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

    const int split = blockIdx.x, g = blockIdx.y, b = b0 + blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile0 = split * tps;
    const int ntiles_all = (L + kTile - 1) / kTile;
    const int ntiles = min(tps, ntiles_all - tile0);
    const int pos_end = min(L, (tile0 + ntiles) * kTile);

    pdl_launch_dependents();  // the combine kernel waits for this grid's completion
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kGroup);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const uint32_t sbase = smem_u32(smem);
    if (warp == kGroup) {
        // ---------------- producer ----------------
        // Positions [0, L) of the cache are not written by the prep kernel of
        // this call (it appends at L), so the loads start at once, before the
        // prep kernel is done.  The one exception is the tile holding position
        // L - 1: the preceding call on this cache appended it, and a fused
        // call (gqa_fused_kernel) lets its successor start before it
        // completes.  That tile is loaded after this grid's wait, which
        // returns once the prep kernel, and so everything before it, is done.
        if (lane == 0) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
            const int zc = b * nkv + g;
            int it = 0;
            bool waited = false;
            for (; it < ntiles; it++) {
                const int st = it % kStages, round = it / kStages;
                if (round > 0 &&
                    !mbar_wait_bounded(smem_u32(&empty[st]), (round - 1) & 1, abort_flag, err))
                    break;
                if (!waited && (tile0 + it) * kTile + kTile > L - 1) {
                    pdl_wait();
                    waited = true;
                }
                const uint32_t fb = smem_u32(&full[st]);
                mbar_arrive_expect_tx(fb, kStageBytes);
                const int p0 = (tile0 + it) * kTile;
                const uint32_t kb = sbase + st * kStageBytes;
#pragma unroll
                for (int sub = 0; sub < 4; sub++) {
                    tma_load_3d(kb + sub * kSubBytes, &tmk, sub * 64, p0, zc, fb);
                    tma_load_3d(kb + kTileBytes + sub * kSubBytes, &tmv, sub * 64, p0, zc, fb);
                }
            }
            // Do not leave while copies this CTA issued may still land.
            for (int j = max(0, it - kStages); j < it; j++)
                mbar_wait_bounded(smem_u32(&full[j % kStages]), (j / kStages) & 1, abort_flag, err);
        }
        return;
    }

    // ---------------- consumers: warp w owns positions [16w, 16w+16) of a tile ----
    const int row = lane >> 2;          // A/C row: head (row & 3), hi/lo (row >> 2)
    const int quad = lane & 3;
    uint32_t qa[16][2];
    pdl_wait();  // q comes from the prep kernel (the producer's K/V loads did not wait)
    {
        const int head = row & 3, hl = row >> 2;
        const uint16_t* qr = q_bf + ((((size_t)b * nkv + g) * kGroup + head) * 2 + hl) * kD;
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + quad * 2);
            qa[kk][1] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 8 + quad * 2);
        }
    }
    float o[32][2];
#pragma unroll
    for (int n = 0; n < 32; n++) o[n][0] = o[n][1] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    attend_tiles(sbase, full, empty, abort_flag, err, qa, tile0, ntiles, pos_end, warp, lane, o, m_run,
                 l_run);

    // ---- fold lo rows into hi rows, then merge the 4 warps through smem ----
#pragma unroll
    for (int n = 0; n < 32; n++) {
        o[n][0] += __shfl_xor_sync(0xffffffffu, o[n][0], 16);
        o[n][1] += __shfl_xor_sync(0xffffffffu, o[n][1], 16);
    }
    named_bar_sync(1, kGroup * 32);  // all consumers are done with the stage buffers
    float* mo = reinterpret_cast<float*>(smem);           // [4 warps][4 heads][256]
    float* mm = mo + kGroup * kGroup * kD;                // [4][4]
    float* ml = mm + kGroup * kGroup;                     // [4][4]
    if (lane < 16) {
        const int head = lane >> 2;
        float* dst = mo + (warp * kGroup + head) * kD + quad * 2;
#pragma unroll
        for (int n = 0; n < 32; n++) {
            dst[n * 8] = o[n][0];
            dst[n * 8 + 1] = o[n][1];
        }
        if (quad == 0) {
            mm[warp * kGroup + head] = m_run;
            ml[warp * kGroup + head] = l_run;
        }
    }
    named_bar_sync(1, kGroup * 32);
    const int t = threadIdx.x;  // 0..127
#pragma unroll
    for (int e = 0; e < (kGroup * kD) / 128; e++) {
        const int idx = e * 128 + t;
        const int head = idx / kD, d = idx % kD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kGroup; w++) M = fmaxf(M, mm[w * kGroup + head]);
        float acc = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kGroup; w++) {
                const float mw = mm[w * kGroup + head];
                const float sc = (mw == -INFINITY) ? 0.f : exp2f((mw - M) * kLog2e);
                acc += sc * mo[(w * kGroup + head) * kD + d];
            }
        }
        const size_t hidx = ((size_t)b * nkv + g) * kGroup + head;
        part_o[(hidx * nsplit + split) * kD + d] = acc;
        if (d == 0) {
            float lsum = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < kGroup; w++) {
                    const float mw = mm[w * kGroup + head];
                    lsum += (mw == -INFINITY) ? 0.f : exp2f((mw - M) * kLog2e) * ml[w * kGroup + head];
                }
            }
            part_ml[(hidx * nsplit + split) * 2 + 0] = M;
            part_ml[(hidx * nsplit + split) * 2 + 1] = lsum;
        }
    }
}

// ---------------------------------------------------------------------------
// 3. combine splits + the new token (f32) + sigmoid gate (gemv.rs:1008-1011)
// One CTA per (sequence, query head): warp w merges splits w, w + 8, ... with
// lane l holding dims [8l, 8l + 8), all of a warp's loads in flight at once;
// then thread d merges the 8 warps' partials and the new token for dim d.
// ---------------------------------------------------------------------------
constexpr int kCombWarps = 8;
constexpr int kCombUnroll = 4;  // splits a warp loads at once

__global__ void __launch_bounds__(256)
gqa_combine_kernel(const float* __restrict__ q_f32, const float* __restrict__ kn,
                   const float* __restrict__ v_new, const float* __restrict__ q_gate,
                   const float* __restrict__ part_o, const float* __restrict__ part_ml, int nsplit,
                   float* __restrict__ out, int kv_lo, int nkv, int b0) {
    // Waits for the attention grid (and, through it, the prep grid).  It never
    // lets its successor start early: the next call's attention kernel loads
    // the cache without waiting, which is safe only once this call is done.
    pdl_wait();
    const int bh = b0 * nkv * kGroup + blockIdx.x;  // (sequence, query head) row of the cache's heads
    const int nh = nkv * kGroup;
    const int b = bh / nh, hl = bh % nh, gl = hl / kGroup;
    const int h = kv_lo * kGroup + hl, g = kv_lo + gl;  // model heads (inputs)
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    __shared__ float s_red[kCombWarps];
    __shared__ __align__(16) float s_o[kCombWarps][kD];
    __shared__ float s_m[kCombWarps], s_l[kCombWarps];

    // the new token's score q . k_new (f32, never rounded for this step)
    float prod = q_f32[(size_t)bh * kD + d] * kn[((size_t)b * nkv + gl) * kD + d];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) prod += __shfl_xor_sync(0xffffffffu, prod, o);
    if (lane == 0) s_red[warp] = prod;

    // this warp's splits, online over groups of kCombUnroll
    const float* ml = part_ml + (size_t)bh * nsplit * 2;
    const float* po = part_o + (size_t)bh * nsplit * kD + 8 * lane;
    float M = -INFINITY, lw = 0.f;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.f;
    for (int i0 = warp; i0 < nsplit; i0 += kCombWarps * kCombUnroll) {
        float mi[kCombUnroll], li[kCombUnroll];
        float4 oa[kCombUnroll], ob[kCombUnroll];
#pragma unroll
        for (int u = 0; u < kCombUnroll; u++) {
            const int i = i0 + u * kCombWarps;
            if (i < nsplit) {
                mi[u] = ml[2 * i];
                li[u] = ml[2 * i + 1];
                oa[u] = reinterpret_cast<const float4*>(po + (size_t)i * kD)[0];
                ob[u] = reinterpret_cast<const float4*>(po + (size_t)i * kD)[1];
            } else {
                mi[u] = -INFINITY;
                li[u] = 0.f;
                oa[u] = ob[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float Mn = M;
#pragma unroll
        for (int u = 0; u < kCombUnroll; u++) Mn = fmaxf(Mn, mi[u]);
        if (Mn == -INFINITY) continue;  // nothing attended yet (empty splits)
        const float c = exp2f((M - Mn) * kLog2e);  // 0 while M is -inf
        lw *= c;
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] *= c;
#pragma unroll
        for (int u = 0; u < kCombUnroll; u++) {
            if (mi[u] == -INFINITY) continue;
            const float w = exp2f((mi[u] - Mn) * kLog2e);
            lw += w * li[u];
            acc[0] += w * oa[u].x; acc[1] += w * oa[u].y; acc[2] += w * oa[u].z; acc[3] += w * oa[u].w;
            acc[4] += w * ob[u].x; acc[5] += w * ob[u].y; acc[6] += w * ob[u].z; acc[7] += w * ob[u].w;
        }
        M = Mn;
    }
    reinterpret_cast<float4*>(&s_o[warp][8 * lane])[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(&s_o[warp][8 * lane])[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (lane == 0) {
        s_m[warp] = M;
        s_l[warp] = lw;
    }
    __syncthreads();
    float s_new = 0.f;
#pragma unroll
    for (int w = 0; w < kCombWarps; w++) s_new += s_red[w];
    float Mall = s_new;
#pragma unroll
    for (int w = 0; w < kCombWarps; w++) Mall = fmaxf(Mall, s_m[w]);
    const float wn = exp2f((s_new - Mall) * kLog2e);
    float o = wn * v_new[((size_t)b * kNumKVH + g) * kD + d];
    float lsum = wn;
#pragma unroll
    for (int w = 0; w < kCombWarps; w++) {
        if (s_m[w] == -INFINITY) continue;
        const float f = exp2f((s_m[w] - Mall) * kLog2e);
        o += f * s_o[w][d];
        lsum += f * s_l[w];
    }
    const float gate = q_gate[((size_t)b * kNumH + h) * 2 * kD + kD + d];
    out[(size_t)bh * kD + d] = (o / lsum) * (1.0f / (1.0f + __expf(-gate)));
}

// ---------------------------------------------------------------------------
// 4. one launch for small batches: prep + split-KV attention + combine.
// A cluster of nsplit CTAs (grid.x, up to 16) owns one (sequence, KV head);
// CTA r streams tiles [r*tps, (r+1)*tps) like gqa_attn, computes the 4 query
// heads' q itself (RMSNorm(1+g), RoPE, 1/16) and keeps its merged partial in
// shared memory.  CTA r owns outputs [r*1024/nsplit, (r+1)*1024/nsplit) of
// the group's 4 x 256: every CTA stores its partial of those outputs (and
// its per-head maximum and sum) into CTA r's shared memory, and after one
// cluster barrier CTA r merges them, adds the new token in f32 and applies
// the sigmoid gate.  CTA 0 appends the new k/v.  No workspace.
//
// Launched with programmatic stream serialisation, and it lets its successor
// start once it has itself waited for its predecessor: a successor that is
// the next decode call then loads its cache tiles while this call runs,
// except the tile holding position L-1, which this call may be writing (the
// append of a call on the same cache); that tile and every input are read
// only after the successor's own wait, i.e. after this grid has completed.
// ---------------------------------------------------------------------------
constexpr int kFusedMaxSplit = 16;                 // CTAs per cluster at most
constexpr int kQbRow = kD + 8;                     // bf16 q row, padded: conflict-free fragment loads
constexpr int kFzQ = kStages * kStageBytes;        // q of the 4 heads, f32 [4][256]
constexpr int kFzQb = kFzQ + kGroup * kD * 4;      // q as bf16 hi / lo [4 heads][2][kQbRow]
constexpr int kFzRecv = kFzQb + kGroup * 2 * kQbRow * 2;  // received partials [nsplit][1024 / nsplit]
constexpr int kFzMl = kFzRecv + kGroup * kD * 4;   // received (m, l) [16][2], then q.k_new [4]
constexpr int kFzBars = kFzMl + (2 * kFusedMaxSplit + 4) * 4;
constexpr int kFusedSmem = kFzBars + 2 * kStages * 8 + 16 + 1024 /*align*/;
// outputs per consumer thread after the merge: 4 x 256 / (nsplit x 128), nsplit >= 2
constexpr int kFusedPerThread = 4;

__global__ void __launch_bounds__(160, 1)
gqa_fused_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                 const float* __restrict__ q_gate, const float* __restrict__ k_new,
                 const float* __restrict__ v_new, const float* __restrict__ q_norm,
                 const float* __restrict__ k_norm, const float* __restrict__ rope_cos,
                 const float* __restrict__ rope_sin, int64_t pos, uint16_t* __restrict__ kcache,
                 uint16_t* __restrict__ vcache, int cap, const float* __restrict__ c_gate,
                 const float* __restrict__ c_v, float* __restrict__ out, int tps, int kv_lo, int nkv,
                 int b0, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* q_s = reinterpret_cast<float*>(smem + kFzQ);
    uint16_t* q_b = reinterpret_cast<uint16_t*>(smem + kFzQb);
    float* recv_o = reinterpret_cast<float*>(smem + kFzRecv);
    float* recv_ml = reinterpret_cast<float*>(smem + kFzMl);
    float* s_new = recv_ml + 2 * kFusedMaxSplit;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kFzBars);
    uint64_t* empty = full + kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

    const int split = blockIdx.x, nsplit = gridDim.x;  // split == rank in the cluster
    const int gl = blockIdx.y, g = kv_lo + gl, b = b0 + blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int L = (int)pos;  // cached positions; the new token goes to index L
    const int tile0 = split * tps;
    const int ntiles_all = (L + kTile - 1) / kTile;
    const int ntiles = max(0, min(tps, ntiles_all - tile0));
    const int pos_end = min(L, (tile0 + ntiles) * kTile);
    const int per = (kGroup * kD) / nsplit;  // outputs this CTA produces after the merge
    float red_gate[kFusedPerThread], red_v[kFusedPerThread];

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kGroup);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // every CTA of the cluster has started before any stores into another's
    // shared memory (the matching wait comes just before the first such store)
    cluster_arrive_relaxed();
    const uint32_t sbase = smem_u32(smem);

    if (warp == kGroup) {
        // ---------------- producer warp ----------------
        const int zc = b * nkv + gl;
        auto issue = [&](int it) {
            const int st = it % kStages;
            const uint32_t fb = smem_u32(&full[st]);
            mbar_arrive_expect_tx(fb, kStageBytes);
            const int p0 = (tile0 + it) * kTile;
            const uint32_t kb = sbase + st * kStageBytes;
#pragma unroll
            for (int sub = 0; sub < 4; sub++) {
                tma_load_3d(kb + sub * kSubBytes, &tmk, sub * 64, p0, zc, fb);
                tma_load_3d(kb + kTileBytes + sub * kSubBytes, &tmv, sub * 64, p0, zc, fb);
            }
        };
        int it = 0;
        if (lane == 0) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
            // before the wait: the first ring's tiles whose positions all lie below L - 1,
            // and the later such tiles into L2 (their ring slots free up only after it)
            for (; it < min(ntiles, kStages); it++) {
                if ((tile0 + it) * kTile + kTile > L - 1) break;
                issue(it);
            }
            if (it == kStages) {
                const size_t plane = ((size_t)b * nkv + gl) * cap;
                for (int j = kStages; j < ntiles; j++) {
                    const int p0 = (tile0 + j) * kTile;
                    if (p0 + kTile > L - 1) break;
                    bulk_prefetch_l2(kcache + (plane + p0) * kD, kTile * kD * 2);
                    bulk_prefetch_l2(vcache + (plane + p0) * kD, kTile * kD * 2);
                }
            }
        }
        it = __shfl_sync(0xffffffffu, it, 0);
        // the layer's parameters are read before the wait (they are not outputs of
        // the preceding kernel), the new token's k only after it
        float kn[8];
#pragma unroll
        for (int i = 0; i < 8; i++) kn[i] = k_norm[lane + 32 * i];
        const float c = rope_cos[pos * kHalfRot + lane];
        const float s = rope_sin[pos * kHalfRot + lane];
        pdl_wait();
        // the new token's k: RMSNorm(1+g) + partial RoPE (gemv.rs:945-955); CTA 0 appends k, v
        {
            const float* src = k_new + ((size_t)b * kNumKVH + g) * kD;
            float x[8];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                x[i] = src[lane + 32 * i];
                ss = fmaf(x[i], x[i], ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.0f / sqrtf(ss * (1.0f / kD) + 1e-6f);  // gemv.rs:591
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = x[i] * inv * (1.0f + kn[i]);
            const float x1 = x[0], x2 = x[1];
            x[0] = x1 * c - x2 * s;
            x[1] = x2 * c + x1 * s;
            // the new token's score q . k_new (f32) of the 4 heads, once their q is in
            // shared memory (the consumers arrive on barrier 2 after writing it)
            named_bar_sync(2, 5 * 32);
#pragma unroll
            for (int h = 0; h < kGroup; h++) {
                float prod = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) prod = fmaf(q_s[h * kD + lane + 32 * i], x[i], prod);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) prod += __shfl_xor_sync(0xffffffffu, prod, o);
                if (lane == 0) s_new[h] = prod;
            }
            if (split == 0) {
                const size_t row = (((size_t)b * nkv + gl) * cap + pos) * kD;
                const float* vs = v_new + ((size_t)b * kNumKVH + g) * kD;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int e = lane + 32 * i;
                    kcache[row + e] = bf16_bits_rn(x[i]);
                    vcache[row + e] = bf16_bits_rn(vs[e]);
                }
            }
        }
        if (lane == 0) {
            for (; it < ntiles; it++) {
                const int round = it / kStages;
                if (round > 0 &&
                    !mbar_wait_bounded(smem_u32(&empty[it % kStages]), (round - 1) & 1, abort_flag, err))
                    break;
                issue(it);
            }
            // every copy this CTA issued has landed before the ring is reused below
            for (int j = max(0, it - kStages); j < it; j++)
                mbar_wait_bounded(smem_u32(&full[j % kStages]), (j / kStages) & 1, abort_flag, err);
        }
        __syncwarp();
        cluster_wait();
    } else {
        // ---------------- consumers ----------------
        {   // warm L2 with this call's small inputs before the wait (a prefetch
            // reads nothing into registers, so it cannot see stale data)
            const int t = threadIdx.x;
            const float* qg = q_gate + ((size_t)b * kNumH + g * kGroup) * 2 * kD;  // 4 heads, 8 KB
            if (t < 64) prefetch_l2(qg + t * 32);
            else if (t < 72) prefetch_l2(q_norm + (t - 64) * 32);
            else if (t < 80) prefetch_l2(k_norm + (t - 72) * 32);
            else if (t < 88) prefetch_l2(k_new + ((size_t)b * kNumKVH + g) * kD + (t - 80) * 32);
            else if (t < 96) prefetch_l2(c_v + ((size_t)b * kNumKVH + g) * kD + (t - 88) * 32);
            else if (t == 96) prefetch_l2(rope_cos + pos * kHalfRot);
            else if (t == 97) prefetch_l2(rope_sin + pos * kHalfRot);
            else if (c_gate != q_gate && t < 98 + 32)
                prefetch_l2(c_gate + ((size_t)b * kNumH + g * kGroup + (t - 98) / 8) * 2 * kD + kD + ((t - 98) % 8) * 32);
        }
        // the layer's parameters before the wait (not outputs of the preceding kernel)
        float qn[8];
#pragma unroll
        for (int i = 0; i < 8; i++) qn[i] = q_norm[lane + 32 * i];
        const float rc = rope_cos[pos * kHalfRot + lane];
        const float rs = rope_sin[pos * kHalfRot + lane];
        pdl_wait();  // q comes from the preceding kernel
        pdl_launch_dependents();
        // the gate logit and new v of the outputs this thread produces after
        // the cluster merge, loaded now so they arrive while the tiles stream
#pragma unroll
        for (int u = 0; u < kFusedPerThread; u++) {
            const int oi = threadIdx.x + u * (kGroup * 32);
            if (oi >= per) break;
            const int idx = split * per + oi;
            const int head = idx / kD, d = idx % kD;
            red_gate[u] = c_gate[((size_t)b * kNumH + g * kGroup + head) * 2 * kD + kD + d];
            red_v[u] = c_v[((size_t)b * kNumKVH + g) * kD + d];
        }
        // q of query head g*4 + warp: RMSNorm(1+g), RoPE, scale 1/16 (gemv.rs:945-959), as in gqa_prep
        {
            const int h = g * kGroup + warp;
            const float* src = q_gate + ((size_t)b * kNumH + h) * 2 * kD;
            float x[8];
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                x[i] = src[lane + 32 * i];
                ss = fmaf(x[i], x[i], ss);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.0f / sqrtf(ss * (1.0f / kD) + 1e-6f);
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = x[i] * inv * (1.0f + qn[i]);
            const float x1 = x[0], x2 = x[1];
            x[0] = x1 * rc - x2 * rs;
            x[1] = x2 * rc + x1 * rs;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int e = lane + 32 * i;
                const float qs = x[i] * 0.0625f;  // scale 1/sqrt(256), exact
                const uint16_t hi = bf16_bits_rn(qs);
                q_s[warp * kD + e] = qs;
                q_b[(warp * 2 + 0) * kQbRow + e] = hi;
                q_b[(warp * 2 + 1) * kQbRow + e] = bf16_bits_rn(qs - bf16_bits_to_f32(hi));
            }
        }
        named_bar_sync(1, kGroup * 32);
        asm volatile("bar.arrive 2, %0;" ::"n"(5 * 32) : "memory");  // q_s is ready for the producer warp
        const int row = lane >> 2, quad = lane & 3;
        uint32_t qa[16][2];
        {   // column row & 3 (head), hi (row < 4) or lo
            const uint16_t* qr = q_b + ((row & 3) * 2 + (row >> 2)) * kQbRow;
#pragma unroll
            for (int kk = 0; kk < 16; kk++) {
                qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + quad * 2);
                qa[kk][1] = *reinterpret_cast<const uint32_t*>(qr + kk * 16 + 8 + quad * 2);
            }
        }
        float oc[16][4];
#pragma unroll
        for (int mt = 0; mt < 16; mt++) oc[mt][0] = oc[mt][1] = oc[mt][2] = oc[mt][3] = 0.f;
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
        attend_tiles_t(sbase, full, empty, abort_flag, err, qa, tile0, ntiles, pos_end, warp, lane, oc, m_run,
                       l_run);
        // hi + lo columns: lanes q and q ^ 2 (q < 2 keeps the sums)
#pragma unroll
        for (int mt = 0; mt < 16; mt++)
#pragma unroll
            for (int k = 0; k < 4; k++) oc[mt][k] += __shfl_xor_sync(0xffffffffu, oc[mt][k], 2);
        named_bar_sync(1, kGroup * 32);  // all consumers are done with the stage buffers
        // the 4 warps' partials, rows padded by 8 floats so a store instruction's
        // 16 lanes (4 heads' rows apart) fall on distinct banks
        constexpr int kRow = kD + 8;
        float* mo = reinterpret_cast<float*>(smem);  // [4 warps][4 heads][kRow]
        float* mm = mo + kGroup * kGroup * kRow;     // [4][4]
        float* ml = mm + kGroup * kGroup;            // [4][4]
        float* sc = ml + kGroup * kGroup;            // [4][4] scale of warp w's partial of head h
        if (quad < 2) {  // heads 2q, 2q + 1 at dims 16mt + lane/4 (+8)
            const int g8 = lane >> 2;
            float* d0 = mo + (warp * kGroup + 2 * quad) * kRow + g8;
            float* d1 = d0 + kRow;
#pragma unroll
            for (int mt = 0; mt < 16; mt++) {
                d0[mt * 16] = oc[mt][0];
                d1[mt * 16] = oc[mt][1];
                d0[mt * 16 + 8] = oc[mt][2];
                d1[mt * 16 + 8] = oc[mt][3];
            }
            if (g8 == 0) {
                mm[warp * kGroup + 2 * quad] = m_run[0];
                mm[warp * kGroup + 2 * quad + 1] = m_run[1];
                ml[warp * kGroup + 2 * quad] = l_run[0];
                ml[warp * kGroup + 2 * quad + 1] = l_run[1];
            }
        }
        named_bar_sync(1, kGroup * 32);
        cluster_wait();
        const int t = threadIdx.x;  // 0..127
        if (t < kGroup) {  // head t: the CTA's maximum, sum and the 4 warps' scales
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kGroup; w++) M = fmaxf(M, mm[w * kGroup + t]);
            float lsum = 0.f;
#pragma unroll
            for (int w = 0; w < kGroup; w++) {
                const float mw = mm[w * kGroup + t];
                const float f = (mw == -INFINITY) ? 0.f : exp2f((mw - M) * kLog2e);
                sc[w * kGroup + t] = f;
                lsum += f * ml[w * kGroup + t];
            }
            // (m, l) of head t to the CTAs that own its outputs
            for (int r = t * kD / per; r < (t + 1) * kD / per; r++)
                st_dsmem_v2(recv_ml + 2 * split, (uint32_t)r, M, (M == -INFINITY) ? 0.f : lsum);
        }
        named_bar_sync(1, kGroup * 32);
        // this CTA's merged partial: output idx goes to CTA idx / per, which
        // receives every CTA's partial of its outputs [nsplit][per]; four
        // adjacent outputs a thread (one owner: per is a multiple of 4), one
        // 16-byte store into the owner's shared memory
        static_assert((kGroup * kD) % (4 * 128) == 0 && (kGroup * kD / kFusedMaxSplit) % 4 == 0,
                      "four outputs a thread, never split between owners");
#pragma unroll
        for (int e = 0; e < (kGroup * kD) / (4 * 128); e++) {
            const int idx = 4 * (e * 128 + t);
            const int head = idx / kD, d = idx % kD;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int w = 0; w < kGroup; w++) {
                const float f = sc[w * kGroup + head];
                const float4 m = *reinterpret_cast<const float4*>(&mo[(w * kGroup + head) * kRow + d]);
                acc.x = fmaf(f, m.x, acc.x);
                acc.y = fmaf(f, m.y, acc.y);
                acc.z = fmaf(f, m.z, acc.z);
                acc.w = fmaf(f, m.w, acc.w);
            }
            st_dsmem_v4(recv_o + split * per + idx % per, (uint32_t)(idx / per), acc);
        }
    }
    // every CTA's pushes have landed (and s_new, written by the producer warp, is visible)
    cluster_sync_all();
    // outputs [split*per, (split+1)*per) of the group's 4 x 256, thread t
    // taking t, t + 128, ...: merge the nsplit partials, add the new token,
    // apply the gate (gemv.rs:1008-1011)
    if (warp < kGroup) {
        // every output of this CTA belongs to one head (per divides 256): warp 0
        // forms the head's maximum, the splits' weights and the sum once, in a
        // fixed order; the stage buffers hold them (free since the pushes)
        static_assert(kD % (kGroup * kD / kFusedMaxSplit) == 0 && kFusedMaxSplit <= 31, "one head per owner");
        float* wsc = reinterpret_cast<float*>(smem);  // [i < nsplit]: split weights, [31]: new token, [30]: sum
        const int head = (split * per) / kD;
        if (warp == 0) {
            const float sn = s_new[head];
            const bool in = lane < nsplit;
            const float mi = in ? recv_ml[2 * lane] : -INFINITY;
            const float li = in ? recv_ml[2 * lane + 1] : 0.f;
            float M = fmaxf(sn, mi);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float f = (mi == -INFINITY) ? 0.f : exp2f((mi - M) * kLog2e);
            float ls = f * li;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
            const float wn = exp2f((sn - M) * kLog2e);
            if (in) wsc[lane] = f;
            if (lane == 0) {
                wsc[31] = wn;
                wsc[30] = ls + wn;
            }
        }
        named_bar_sync(1, kGroup * 32);
#pragma unroll
        for (int u = 0; u < kFusedPerThread; u++) {
            const int oi = threadIdx.x + u * (kGroup * 32);
            if (oi >= per) break;
            const int d = (split * per + oi) % kD;
            float acc = wsc[31] * red_v[u];
#pragma unroll
            for (int i = 0; i < kFusedMaxSplit; i++)
                if (i < nsplit) acc = fmaf(wsc[i], recv_o[i * per + oi], acc);
            out[(((size_t)b * nkv + gl) * kGroup + head) * kD + d] =
                (acc / wsc[30]) * (1.0f / (1.0f + __expf(-red_gate[u])));
        }
    }
}

}  // namespace

// Workspace of a call on sequences [b0, b0 + nb) of a batch-`batch` cache
// (nb = batch: the whole batch).
size_t gqa_decode_ws_bytes(int batch, int nkv, int64_t seq_len, int num_sms, int nb) {
    Plan p = plan_for(nb < 0 ? batch : nb, nkv, seq_len, num_sms);
    return ws_layout(batch, nkv, p.nsplit).total;
}

// CTAs per cluster of the fused kernel on this device: 16 where a cluster of
// 16 such CTAs can be resident (a non-portable size), else 8; 0 if neither.
// Decided once per device, so every call on a device merges its splits in
// the same order.
static int fused_splits(qm_ctx* ctx) {
    static std::atomic<int> known[64];
    const int dev = ctx->device;
    if (dev >= 0 && dev < 64) {
        const int k = known[dev].load(std::memory_order_acquire);
        if (k != 0) return k > 0 ? k : 0;
    }
    int found = -1;
    if (cudaFuncSetAttribute(gqa_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmem) ==
            cudaSuccess &&
        cudaFuncSetAttribute(gqa_fused_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
            cudaSuccess) {
        for (int S : {16, 8}) {
            cudaLaunchConfig_t c = {};
            c.gridDim = dim3(S, 1, 1);
            c.blockDim = dim3(160);
            c.dynamicSmemBytes = kFusedSmem;
            cudaLaunchAttribute a[1];
            a[0].id = cudaLaunchAttributeClusterDimension;
            a[0].val.clusterDim.x = S;
            a[0].val.clusterDim.y = 1;
            a[0].val.clusterDim.z = 1;
            c.attrs = a;
            c.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, gqa_fused_kernel, &c) == cudaSuccess && n >= 1) {
                found = S;
                break;
            }
        }
    }
    cudaGetLastError();  // a refused query leaves no sticky error behind
    if (dev >= 0 && dev < 64) known[dev].store(found, std::memory_order_release);
    return found > 0 ? found : 0;
}

// The fused kernel serves calls whose clusters fit in one wave and whose
// context is short enough that a cluster's CTAs stream it as fast as the
// three-kernel grid would.  QORA_MIXER_GQA_FUSED=0 turns it off, =1 drops the
// context limit (tuning and tests).
constexpr int kFusedAutoMaxTiles = 256;  // L <= 16384

static bool use_fused(qm_ctx* ctx, int B, int nkv, int64_t L, int S) {
    static const int mode = [] {
        const char* e = getenv("QORA_MIXER_GQA_FUSED");
        return e ? atoi(e) : -1;
    }();
    if (mode == 0 || S == 0) return false;
    if ((int64_t)B * nkv * S > ctx->num_sms) return false;
    return mode == 1 || (L + kTile - 1) / kTile <= kFusedAutoMaxTiles;
}

cudaError_t launch_gqa_decode(qm_ctx* ctx, const qm_gqa_params* prm, qm_kv* kv,
                              const float* q_gate, const float* k_new, const float* v_new,
                              float* out, void* ws, size_t ws_bytes, int b0, int nb,
                              const GqaCombineSrc* comb) {
    const int B = nb < 0 ? kv->batch : nb;  // sequences [b0, b0 + B) of the cache
    const int64_t L = kv->seq_len;  // cached positions; the new token goes to index L
    const int nkv = kv->nkv;
    const int S = fused_splits(ctx);
    if (use_fused(ctx, B, nkv, L, S)) {
        const float* c_gate = q_gate;
        const float* c_v = v_new;
        if (comb) {
            if (comb->ready) {
                const cudaError_t e = cudaStreamWaitEvent(ctx->stream, comb->ready, 0);
                if (e != cudaSuccess) return e;
            }
            c_gate = comb->q_gate ? comb->q_gate : q_gate;
            c_v = comb->v_new ? comb->v_new : v_new;
        }
        const int ntiles = (int)((L + kTile - 1) / kTile);
        const int tps = (ntiles + S - 1) / S;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = S;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[1].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t c = {};
        c.gridDim = dim3(S, nkv, B);
        c.blockDim = dim3(160);
        c.dynamicSmemBytes = kFusedSmem;
        c.stream = ctx->stream;
        c.attrs = at;
        c.numAttrs = 2;
        cudaError_t e;
        {
            TimedLaunch tl(ctx, "gqa_fused");
            e = cudaLaunchKernelEx(&c, gqa_fused_kernel, kv->tmap_k, kv->tmap_v, q_gate, k_new, v_new,
                                   prm->q_norm, prm->k_norm, prm->rope_cos, prm->rope_sin, L, kv->k, kv->v,
                                   kv->capacity, c_gate, c_v, out, tps, kv->kv_lo, nkv, b0, ctx->d_err);
        }
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e == cudaSuccess) ctx->launches += 1;
        return e;
    }
    const Plan pl = plan_for(B, nkv, L, ctx->num_sms);
    const WsLayout w = ws_layout(kv->batch, nkv, pl.nsplit);  // indexed by absolute sequence
    if (w.total > ws_bytes) return cudaErrorInvalidValue;
    char* base = static_cast<char*>(ws);
    uint16_t* q_bf = reinterpret_cast<uint16_t*>(base + w.q_bf);
    float* q_f32 = reinterpret_cast<float*>(base + w.q_f32);
    float* kn = reinterpret_cast<float*>(base + w.kn);
    float* part_o = reinterpret_cast<float*>(base + w.part_o);
    float* part_ml = reinterpret_cast<float*>(base + w.part_ml);
    cudaStream_t st = ctx->stream;

    // All three kernels are launched with programmatic stream serialization
    // (each may start while its predecessor runs; see the kernels' waits).
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    auto cfg_for = [&](dim3 grid, int threads, size_t smem) {
        cudaLaunchConfig_t c = {};
        c.gridDim = grid;
        c.blockDim = dim3(threads);
        c.dynamicSmemBytes = smem;
        c.stream = st;
        c.attrs = pdl;
        c.numAttrs = 1;
        return c;
    };
    cudaError_t e;
    {
        TimedLaunch tl(ctx, "gqa_prep");
        const cudaLaunchConfig_t c = cfg_for(dim3(B * nkv), 160, 0);
        e = cudaLaunchKernelEx(&c, gqa_prep_kernel, q_gate, k_new, v_new, prm->q_norm, prm->k_norm,
                               prm->rope_cos, prm->rope_sin, L, kv->k, kv->v, kv->capacity, q_bf, q_f32,
                               kn, kv->kv_lo, nkv, b0);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    if (pl.nsplit > 0) {
        static std::atomic<uint64_t> attr_set{0};
        e = set_smem_once(attr_set, ctx->device, gqa_attn_kernel, kAttnSmem);
        if (e != cudaSuccess) return e;
        TimedLaunch tl(ctx, "gqa_attn");
        const cudaLaunchConfig_t c = cfg_for(dim3(pl.nsplit, nkv, B), 160, kAttnSmem);
        e = cudaLaunchKernelEx(&c, gqa_attn_kernel, kv->tmap_k, kv->tmap_v, (const uint16_t*)q_bf, part_o,
                               part_ml, (int)L, pl.tps, pl.nsplit, nkv, b0, ctx->d_err);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        ctx->launches += 1;
    }
    const float* c_gate = q_gate;
    const float* c_v = v_new;
    if (comb) {
        if (comb->ready) {
            e = cudaStreamWaitEvent(st, comb->ready, 0);
            if (e != cudaSuccess) return e;
        }
        c_gate = comb->q_gate ? comb->q_gate : q_gate;
        c_v = comb->v_new ? comb->v_new : v_new;
    }
    {
        TimedLaunch tl(ctx, "gqa_combine");
        const cudaLaunchConfig_t c = cfg_for(dim3(B * nkv * kGroup), 256, 0);
        e = cudaLaunchKernelEx(&c, gqa_combine_kernel, (const float*)q_f32, (const float*)kn, c_v, c_gate,
                               (const float*)part_o, (const float*)part_ml, pl.nsplit, out, kv->kv_lo,
                               nkv, b0);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) ctx->launches += 1;
    return e;
}

}  // namespace qm
