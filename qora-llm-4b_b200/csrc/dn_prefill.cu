// DeltaNet chunked prefill on the 5th-generation tensor cores.
//
// Replaces the sequential loop of prefill_deltanet_layer, src/gemv.rs:1119-1219
// (and the CPU recurrence that prefill_deltanet_layer_gpu runs between two
// device round trips, src/gpu_inference.rs:464-604).
//
// Per token the reference does S <- a S; S <- S + b (v - S k) k^T; y = S q.
// Over a chunk of C = 64 tokens this is the WY/UT form (G_t = cumulative
// log-decay inside the chunk, g_t = log a_t):
//   A_ts = b_t e^(G_t-G_s) (k_t.k_s)  (s < t),     T = (I + A)^-1
//   W^T  = K^T (T diag(b e^G))^T      U~^T = V^T (T diag(b))^T
//   U^T  = U~^T - S0 W^T
//   Y^T  = diag-scale(e^G) S0 Q^T + U^T P'^T,     P'_ts = e^(G_t-G_s) q_t.k_s (s <= t)
//   S    = e^(G_63) S0 + (U^T diag(e^(G_63-G))) K
// written transposed so that every tensor-core product has M = 128 (the v
// or k dimension) and the f32 state S [v x k] lives in TMEM for the whole
// sequence.  Precision: the outputs are heavy-tailed across heads (slowly
// decaying heads carry large states), so one fp16/bf16 rounding of an
// operand already costs ~1e-2 of max-error/RMS.  Every intra-chunk product
// is therefore compensated — operands split into fp16 hi + lo and
// D = hi.hi + hi.lo + lo.hi (3 MMAs) — and only the two products with the
// state (S0 W^T, S0 Q^T) use a single fp16 rounding; the triangular solve
// runs in f32 on the CUDA cores.
//
// Kernels:
//   dn_prefill_prep   conv1d(k=4)+SiLU, per-head L2 norm (q * 1/sqrt(128)),
//                     log-decay g and beta (gemv.rs:1132-1172), written as fp16
//                     hi/lo planes [B*heads][T][128] + f32 g/beta [B*32][T]
//   dn_conv_ring      stores the last raw inputs into the conv history ring
//   dn_prefill_chunk  one CTA (128 threads) per (sequence, V head), chunks in
//                     order, TMA loads, tcgen05 products, f32 solve
//   dn_prefill_gate   optional per-head RMSNorm * SiLU(z) (gemv.rs:1205-1219)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {

int encode_rows_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                     uint32_t box_inner, uint32_t box_rows, bool fp16);

namespace {

constexpr int kC = 64;  // chunk length (tokens)
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// prep: one CTA per (8-token tile, head-vector, sequence); 128 threads = channels
// head-vectors 0..15 = q heads, 16..31 = k heads, 32..63 = v heads
// ---------------------------------------------------------------------------
constexpr int kPrepTok = 8;

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

__global__ void __launch_bounds__(128)
dn_prefill_prep(const uint16_t* __restrict__ qkv, const float* __restrict__ a_in,
                const float* __restrict__ b_in, const float* __restrict__ conv_w,
                const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                const float* __restrict__ ring, int64_t conv_pos, int T,
                uint16_t* __restrict__ qh, uint16_t* __restrict__ ql, uint16_t* __restrict__ kh,
                uint16_t* __restrict__ kl, uint16_t* __restrict__ vh, uint16_t* __restrict__ vl,
                float* __restrict__ gout, float* __restrict__ bout) {
    const int tile = blockIdx.x, hv = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ch = hv * kHd + tid;  // channel within the 8192 mixed qkv
    const float4 w = reinterpret_cast<const float4*>(conv_w)[ch];
    const uint16_t* xb = qkv + (size_t)b * T * kQKVDim + ch;
    const float* rb = ring + (size_t)b * kConvSlots * kQKVDim + ch;
    const int t0 = tile * kPrepTok;
    auto xval = [&](int t) -> float {  // raw input of token t (negative: history ring)
        if (t >= 0) return bf16_bits_to_f32(xb[(size_t)t * kQKVDim]);
        const int64_t tok = conv_pos + t;
        if (tok < 0) return 0.f;
        return rb[(size_t)(tok & 3) * kQKVDim];
    };
    float x3 = xval(t0 - 3), x2 = xval(t0 - 2), x1 = xval(t0 - 1);
    __shared__ float s_red[kPrepTok][4];
    float act[kPrepTok];
#pragma unroll
    for (int i = 0; i < kPrepTok; i++) {
        const int t = t0 + i;
        const float x0 = (t < T) ? xval(t) : 0.f;
        float cv = x3 * w.x;  // gemv.rs:1134-1139: history oldest first, then x
        cv += x2 * w.y;
        cv += x1 * w.z;
        cv += x0 * w.w;
        act[i] = silu_f(cv);
        x3 = x2;
        x2 = x1;
        x1 = x0;
    }
    const bool is_qk = hv < 2 * kNumQK;
    if (is_qk) {
#pragma unroll
        for (int i = 0; i < kPrepTok; i++) {
            float ss = act[i] * act[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) s_red[i][warp] = ss;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kPrepTok; i++) {
            const float n = sqrtf(s_red[i][0] + s_red[i][1] + s_red[i][2] + s_red[i][3]);
            if (n > 1e-12f) act[i] *= 1.0f / n;  // l2_normalize, gemv.rs:1153-1154
            if (hv < kNumQK) act[i] *= 0.08838834764831845f;  // q * 1/sqrt(128)
        }
    }
    uint16_t *ph, *pl;
    size_t plane;
    if (hv < kNumQK) {
        ph = qh; pl = ql; plane = (size_t)b * kNumQK + hv;
    } else if (hv < 2 * kNumQK) {
        ph = kh; pl = kl; plane = (size_t)b * kNumQK + (hv - kNumQK);
    } else {
        ph = vh; pl = vl; plane = (size_t)b * kNumV + (hv - 2 * kNumQK);
    }
#pragma unroll
    for (int i = 0; i < kPrepTok; i++) {
        const int t = t0 + i;
        if (t < T) {
            const size_t o = (plane * T + t) * kHd + tid;
            const __half hi = __float2half_rn(act[i]);
            ph[o] = __half_as_ushort(hi);
            pl[o] = f16_bits_rn(act[i] - __half2float(hi));
        }
    }
    if (hv >= 2 * kNumQK && tid < kPrepTok) {
        // gates of V head vh for this token (gemv.rs:1171-1172), as log-decay
        const int vhh = hv - 2 * kNumQK, t = t0 + tid;
        if (t < T) {
            const float x = a_in[((size_t)b * T + t) * kNumV + vhh] + dt_bias[vhh];
            const float sp = x > 20.0f ? x : log1pf(__expf(x));
            gout[((size_t)b * kNumV + vhh) * T + t] = -__expf(a_log[vhh]) * sp;
            bout[((size_t)b * kNumV + vhh) * T + t] =
                1.0f / (1.0f + __expf(-b_in[((size_t)b * T + t) * kNumV + vhh]));
        }
    }
}

// conv history: token conv_pos + t lands in slot (conv_pos + t) % 4, last 4 tokens
__global__ void dn_conv_ring(const uint16_t* __restrict__ qkv, float* __restrict__ ring,
                             int64_t conv_pos, int T) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (ch >= kQKVDim) return;
    for (int t = (T > 4 ? T - 4 : 0); t < T; t++)
        ring[((size_t)b * kConvSlots + ((conv_pos + t) & 3)) * kQKVDim + ch] =
            bf16_bits_to_f32(qkv[((size_t)b * T + t) * kQKVDim + ch]);
}

// ---------------------------------------------------------------------------
// chunk kernel
// ---------------------------------------------------------------------------
// shared memory map (offsets from a 1024-aligned base)
constexpr int kOffKQh = 0;                 // [K;Q] hi: 2 boxes of [128 rows x 64] fp16 (16 KB each)
constexpr int kOffKQl = 32768;             // [K;Q] lo
constexpr int kOffVh = 65536;              // V hi: 2 boxes [64 x 64] (8 KB) ; later U^T hi [128x64]
constexpr int kOffVl = 81920;              // V lo                            ; later U^T lo
constexpr int kOffT1h = 98304;             // T' hi [64x64] 8 KB ; later W^T hi [128 x 64] 16 KB
constexpr int kOffT1l = 106496;
constexpr int kOffT2h = 114688;            // T'' hi
constexpr int kOffT2l = 122880;
constexpr int kOffPh = 131072;             // P' hi [64x64]
constexpr int kOffPl = 139264;
constexpr int kOffS = 147456;              // S0 fp16 [128 v x 128 k]: 2 boxes [128 x 64]
constexpr int kOffUDh = 180224;            // (U^T diag D) hi [128 x 64]
constexpr int kOffUDl = 196608;
constexpr int kOffA = 212992;              // A f32 [64][64]
constexpr int kOffMisc = 229376;           // G, beta, g: 3 x 64 f32; barriers
constexpr int kChunkSmem = kOffMisc + 3 * 64 * 4 + 64 + 1024;

// TMEM columns
constexpr uint32_t kTmKQ = 0, kTmW = 64, kTmU = 128, kTmY1 = 192, kTmY2 = 256, kTmS = 384;

constexpr uint32_t kNegA = 1u << 13;
constexpr uint32_t kIdKK = umma_idesc_f16kind(128, 64, false, false, false);   // A K, B K
constexpr uint32_t kIdW = umma_idesc_f16kind(128, 64, true, false, false);     // A MN, B K
constexpr uint32_t kIdSW = umma_idesc_f16kind(128, 64, false, true, false) | kNegA;  // -A . B(MN)
constexpr uint32_t kIdSQ = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUP = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUK = umma_idesc_f16kind(128, 128, false, true, false);   // A K, B MN

__device__ __forceinline__ uint32_t swz(int row, int col) {  // fp16 [rows x 64] tile element
    return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

struct ChunkBars {
    uint64_t load, mma;
    uint32_t tmem_base;
    int abort_flag;
};

__global__ void __launch_bounds__(128, 1)
dn_prefill_chunk(const __grid_constant__ CUtensorMap tqh, const __grid_constant__ CUtensorMap tql,
                 const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
                 const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
                 const float* __restrict__ gin, const float* __restrict__ bin,
                 float* __restrict__ S, float* __restrict__ y, int T, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* sG = reinterpret_cast<float*>(smem + kOffMisc);
    float* sB = sG + 64;
    float* sg = sB + 64;
    ChunkBars* bars = reinterpret_cast<ChunkBars*>(sg + 64);
    float* Amat = reinterpret_cast<float*>(smem + kOffA);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sb = smem_u32(smem);

    const int vh = blockIdx.x, b = blockIdx.y, qk = vh >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    const int row = tid;  // TMEM lane == thread (warp w owns lanes 32w..32w+31)

    if (tid == 0) {
        mbar_init(smem_u32(&bars->load), 1);
        mbar_init(smem_u32(&bars->mma), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = bars->tmem_base;

    // ---- initial state: global f32 -> TMEM (master) and fp16 operand copy ----
    float* Sg = S + ((size_t)b * kNumV + vh) * kHd * kHd;
    {
        const float* srow = Sg + (size_t)row * kHd;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = srow[c * 32 + i];
            tmem_st32(tm + lane_addr + kTmS + c * 32, v);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const int k = c * 32 + i;
                *reinterpret_cast<uint32_t*>(smem + kOffS + (k >> 6) * 16384 + swz(row, k & 63)) =
                    pack_bf16(f16_bits_rn(v[i]), f16_bits_rn(v[i + 1]));
            }
        }
        tmem_st_wait();
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();

    uint32_t load_phase = 0, mma_phase = 0;
    bool ok = true;
    // every decision to stop is block-uniform, so no thread skips a barrier
    auto wait_mma = [&]() {
        const bool w = mbar_wait_bounded(smem_u32(&bars->mma), mma_phase, abort_flag, err);
        ok = __syncthreads_and(ok && w) != 0;
        mma_phase ^= 1;
        tc_fence_after();
    };
    auto commit_mma = [&]() {
        if (tid == 0) umma_commit(smem_u32(&bars->mma));
    };
    const size_t plane_qk = (size_t)b * kNumQK + qk, plane_v = (size_t)b * kNumV + vh;
    const int nchunks = (T + kC - 1) / kC;

    for (int ci = 0; ci < nchunks && ok; ci++) {
        const int t0 = ci * kC;
        const int tc = min(kC, T - t0);
        // ---- loads: K/Q/V hi+lo tiles via TMA, gates by threads ----
        if (tid == 0) {
            const uint32_t lb = smem_u32(&bars->load);
            mbar_arrive_expect_tx(lb, 12 * 8192);
            for (int hb = 0; hb < 2; hb++) {  // k halves
                tma_load_3d(sb + kOffKQh + hb * 16384, &tkh, hb * 64, t0, (int)plane_qk, lb);
                tma_load_3d(sb + kOffKQl + hb * 16384, &tkl, hb * 64, t0, (int)plane_qk, lb);
                tma_load_3d(sb + kOffKQh + hb * 16384 + 8192, &tqh, hb * 64, t0, (int)plane_qk, lb);
                tma_load_3d(sb + kOffKQl + hb * 16384 + 8192, &tql, hb * 64, t0, (int)plane_qk, lb);
                tma_load_3d(sb + kOffVh + hb * 8192, &tvh, hb * 64, t0, (int)plane_v, lb);
                tma_load_3d(sb + kOffVl + hb * 8192, &tvl, hb * 64, t0, (int)plane_v, lb);
            }
        }
        if (tid < kC) {
            const bool valid = tid < tc;
            sg[tid] = valid ? gin[plane_v * T + t0 + tid] : 0.f;
            sB[tid] = valid ? bin[plane_v * T + t0 + tid] : 0.f;
        }
        __syncthreads();
        if (warp == 0) {  // inclusive cumulative log-decay G_t
            float g0 = sg[lane], g1 = sg[lane + 32];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u0 = __shfl_up_sync(0xffffffffu, g0, o);
                const float u1 = __shfl_up_sync(0xffffffffu, g1, o);
                if (lane >= o) {
                    g0 += u0;
                    g1 += u1;
                }
            }
            const float tot0 = __shfl_sync(0xffffffffu, g0, 31);
            sG[lane] = g0;
            sG[lane + 32] = g1 + tot0;
        }
        {
            const bool w = mbar_wait_bounded(smem_u32(&bars->load), load_phase, abort_flag, err);
            ok = __syncthreads_and(ok && w) != 0;
        }
        load_phase ^= 1;
        if (!ok) break;

        // ---- MMA1: [K;Q] K^T  (compensated) -> TMEM KQ ----
        if (tid == 0) {
            tc_fence_after();
            int n = 0;
            for (int term = 0; term < 3; term++) {
                const uint32_t abase = sb + (term == 2 ? kOffKQl : kOffKQh);
                const uint32_t bbase = sb + (term == 1 ? kOffKQl : kOffKQh);
                for (int kk = 0; kk < 8; kk++, n++) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16_ss(tm + kTmKQ, umma_sdesc(abase + off, 16, 1024),
                                 umma_sdesc(bbase + off, 16, 1024), kIdKK, n > 0);
                }
            }
        }
        commit_mma();
        wait_mma();
        if (!ok) break;

        // ---- A matrix (rows 0..63) and P' (rows 64..127) from TMEM ----
        {
            float kq[64];
            tmem_ld32(tm + lane_addr + kTmKQ, kq);
            tmem_ld32(tm + lane_addr + kTmKQ + 32, kq + 32);
            tmem_ld_wait();
            if (row < kC) {
                const int t = row;
                const float Gt = sG[t], bt = sB[t];
#pragma unroll
                for (int s = 0; s < kC; s++)
                    Amat[t * kC + s] = (s < t) ? bt * exp2f((Gt - sG[s]) * kLog2e) * kq[s] : 0.f;
            } else {
                const int t = row - kC;
                const float Gt = sG[t];
#pragma unroll
                for (int s = 0; s < kC; s += 2) {
                    const float p0 = (s <= t) ? exp2f((Gt - sG[s]) * kLog2e) * kq[s] : 0.f;
                    const float p1 = (s + 1 <= t) ? exp2f((Gt - sG[s + 1]) * kLog2e) * kq[s + 1] : 0.f;
                    const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
                    *reinterpret_cast<uint32_t*>(smem + kOffPh + swz(t, s)) =
                        pack_bf16(__half_as_ushort(h0), __half_as_ushort(h1));
                    *reinterpret_cast<uint32_t*>(smem + kOffPl + swz(t, s)) =
                        pack_bf16(f16_bits_rn(p0 - __half2float(h0)), f16_bits_rn(p1 - __half2float(h1)));
                }
            }
        }
        tc_fence_before();
        __syncthreads();

        // ---- T = (I + A)^-1, one column per thread (f32); T' = T diag(b e^G), T'' = T diag(b) ----
        if (tid < kC) {
            const int j = tid;
            float tcol[kC];
#pragma unroll
            for (int t = 0; t < kC; t++) {
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                const float* arow = Amat + t * kC;
#pragma unroll
                for (int s = 0; s + 3 < t; s += 4) {
                    const float4 av = *reinterpret_cast<const float4*>(arow + s);
                    a0 = fmaf(av.x, tcol[s], a0);
                    a1 = fmaf(av.y, tcol[s + 1], a1);
                    a2 = fmaf(av.z, tcol[s + 2], a2);
                    a3 = fmaf(av.w, tcol[s + 3], a3);
                }
#pragma unroll
                for (int s = (t / 4) * 4; s < t; s++) a0 = fmaf(arow[s], tcol[s], a0);
                tcol[t] = (t == j) ? 1.f : -((a0 + a1) + (a2 + a3));
            }
            const float bj = sB[j];
            const float c1 = bj * exp2f(sG[j] * kLog2e), c2 = bj;
#pragma unroll
            for (int t = 0; t < kC; t++) {
                const float v1 = tcol[t] * c1, v2 = tcol[t] * c2;
                const __half h1 = __float2half_rn(v1), h2 = __float2half_rn(v2);
                const uint32_t o = swz(t, j);
                *reinterpret_cast<uint16_t*>(smem + kOffT1h + o) = __half_as_ushort(h1);
                *reinterpret_cast<uint16_t*>(smem + kOffT1l + o) = f16_bits_rn(v1 - __half2float(h1));
                *reinterpret_cast<uint16_t*>(smem + kOffT2h + o) = __half_as_ushort(h2);
                *reinterpret_cast<uint16_t*>(smem + kOffT2l + o) = f16_bits_rn(v2 - __half2float(h2));
            }
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();

        // ---- MMA2: W^T = K^T T'^T ; MMA3: U~^T = V^T T''^T (compensated) ; MMA5: Y1 = S0 Q^T ----
        if (tid == 0) {
            tc_fence_after();
            int n = 0;
            for (int term = 0; term < 3; term++) {
                const uint32_t ka = sb + (term == 2 ? kOffKQl : kOffKQh);
                const uint32_t tb = sb + (term == 1 ? kOffT1l : kOffT1h);
                for (int kk = 0; kk < 4; kk++, n++)
                    umma_bf16_ss(tm + kTmW, umma_sdesc(ka + kk * 2048, 16384, 1024),
                                 umma_sdesc(tb + kk * 32, 16, 1024), kIdW, n > 0);
            }
            n = 0;
            for (int term = 0; term < 3; term++) {
                const uint32_t va = sb + (term == 2 ? kOffVl : kOffVh);
                const uint32_t tb = sb + (term == 1 ? kOffT2l : kOffT2h);
                for (int kk = 0; kk < 4; kk++, n++)
                    umma_bf16_ss(tm + kTmU, umma_sdesc(va + kk * 2048, 8192, 1024),
                                 umma_sdesc(tb + kk * 32, 16, 1024), kIdW, n > 0);
            }
            for (int kk = 0; kk < 8; kk++) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tm + kTmY1, umma_sdesc(sb + kOffS + off, 16, 1024),
                             umma_sdesc(sb + kOffKQh + 8192 + off, 16, 1024), kIdSQ, kk > 0);
            }
        }
        commit_mma();
        wait_mma();
        if (!ok) break;

        // ---- W^T (TMEM, lane k) -> fp16 [k][t] for the state product ----
        {
            float wv[64];
            tmem_ld32(tm + lane_addr + kTmW, wv);
            tmem_ld32(tm + lane_addr + kTmW + 32, wv + 32);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < kC; t += 2)
                *reinterpret_cast<uint32_t*>(smem + kOffT1h + swz(row, t)) =
                    pack_bf16(f16_bits_rn(wv[t]), f16_bits_rn(wv[t + 1]));
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();

        // ---- MMA4: U^T -= S0 W^T ----
        if (tid == 0) {
            tc_fence_after();
            for (int kk = 0; kk < 8; kk++) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tm + kTmU, umma_sdesc(sb + kOffS + off, 16, 1024),
                             umma_sdesc(sb + kOffT1h + kk * 2048, 8192, 1024), kIdSW, 1u);
            }
        }
        commit_mma();
        wait_mma();
        if (!ok) break;

        // ---- U^T (lane v) -> hi/lo fp16 [v][s]; U^T diag(D) -> hi/lo; S *= e^G63 ----
        {
            const float G63 = sG[kC - 1];
            float uv[64];
            tmem_ld32(tm + lane_addr + kTmU, uv);
            tmem_ld32(tm + lane_addr + kTmU + 32, uv + 32);
            tmem_ld_wait();
#pragma unroll
            for (int s = 0; s < kC; s += 2) {
                const uint32_t o = swz(row, s);
                const __half h0 = __float2half_rn(uv[s]), h1 = __float2half_rn(uv[s + 1]);
                *reinterpret_cast<uint32_t*>(smem + kOffVh + o) = pack_bf16(__half_as_ushort(h0), __half_as_ushort(h1));
                *reinterpret_cast<uint32_t*>(smem + kOffVl + o) =
                    pack_bf16(f16_bits_rn(uv[s] - __half2float(h0)), f16_bits_rn(uv[s + 1] - __half2float(h1)));
                const float d0 = uv[s] * exp2f((G63 - sG[s]) * kLog2e);
                const float d1 = uv[s + 1] * exp2f((G63 - sG[s + 1]) * kLog2e);
                const __half e0 = __float2half_rn(d0), e1 = __float2half_rn(d1);
                *reinterpret_cast<uint32_t*>(smem + kOffUDh + o) = pack_bf16(__half_as_ushort(e0), __half_as_ushort(e1));
                *reinterpret_cast<uint32_t*>(smem + kOffUDl + o) =
                    pack_bf16(f16_bits_rn(d0 - __half2float(e0)), f16_bits_rn(d1 - __half2float(e1)));
            }
            const float decay = exp2f(G63 * kLog2e);
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float sv[32];
                tmem_ld32(tm + lane_addr + kTmS + c * 32, sv);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) sv[i] *= decay;
                tmem_st32(tm + lane_addr + kTmS + c * 32, sv);
            }
            tmem_st_wait();
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();

        // ---- MMA6: Y2 = U^T P'^T ; MMA7: S += (U^T D) K  (compensated) ----
        if (tid == 0) {
            tc_fence_after();
            int n = 0;
            for (int term = 0; term < 3; term++) {
                const uint32_t ua = sb + (term == 2 ? kOffVl : kOffVh);
                const uint32_t pb = sb + (term == 1 ? kOffPl : kOffPh);
                for (int kk = 0; kk < 4; kk++, n++)
                    umma_bf16_ss(tm + kTmY2, umma_sdesc(ua + kk * 32, 16, 1024),
                                 umma_sdesc(pb + kk * 32, 16, 1024), kIdUP, n > 0);
            }
            for (int term = 0; term < 3; term++) {
                const uint32_t ua = sb + (term == 2 ? kOffUDl : kOffUDh);
                const uint32_t kb = sb + (term == 1 ? kOffKQl : kOffKQh);
                for (int kk = 0; kk < 4; kk++)
                    umma_bf16_ss(tm + kTmS, umma_sdesc(ua + kk * 32, 16, 1024),
                                 umma_sdesc(kb + kk * 2048, 16384, 1024), kIdUK, 1u);
            }
        }
        commit_mma();
        wait_mma();
        if (!ok) break;

        // ---- outputs y_t = e^G_t Y1 + Y2 (lane v); new S -> fp16 operand copy ----
        {
            float y1[64], y2[64];
            tmem_ld32(tm + lane_addr + kTmY1, y1);
            tmem_ld32(tm + lane_addr + kTmY1 + 32, y1 + 32);
            tmem_ld32(tm + lane_addr + kTmY2, y2);
            tmem_ld32(tm + lane_addr + kTmY2 + 32, y2 + 32);
            tmem_ld_wait();
            float* yb = y + ((size_t)b * T + t0) * kVDim + (size_t)vh * kHd + row;
#pragma unroll
            for (int t = 0; t < kC; t++)
                if (t < tc) yb[(size_t)t * kVDim] = exp2f(sG[t] * kLog2e) * y1[t] + y2[t];
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float sv[32];
                tmem_ld32(tm + lane_addr + kTmS + c * 32, sv);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const int k = c * 32 + i;
                    *reinterpret_cast<uint32_t*>(smem + kOffS + (k >> 6) * 16384 + swz(row, k & 63)) =
                        pack_bf16(f16_bits_rn(sv[i]), f16_bits_rn(sv[i + 1]));
                }
            }
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();
    }

    // ---- final state back to global (f32) ----
    if (ok) {
        float* srow = Sg + (size_t)row * kHd;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
            float sv[32];
            tmem_ld32(tm + lane_addr + kTmS + c * 32, sv);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(srow + c * 32 + i) = make_float4(sv[i], sv[i + 1], sv[i + 2], sv[i + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, 512);
    }
}

// per-head RMSNorm (plain gamma) * SiLU(z): one warp per (token, head)
__global__ void dn_prefill_gate(const float* __restrict__ y, const float* __restrict__ z,
                                const float* __restrict__ gamma, float* __restrict__ out,
                                size_t nheads_total) {
    const size_t wid = (size_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (wid >= nheads_total) return;
    const float4 v = reinterpret_cast<const float4*>(y + wid * kHd)[lane];
    float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / kHd) + 1e-6f);
    const float4 zz = reinterpret_cast<const float4*>(z + wid * kHd)[lane];
    const float4 gg = reinterpret_cast<const float4*>(gamma)[lane];
    float4 o;
    o.x = v.x * inv * gg.x * silu_f(zz.x);
    o.y = v.y * inv * gg.y * silu_f(zz.y);
    o.z = v.z * inv * gg.z * silu_f(zz.z);
    o.w = v.w * inv * gg.w * silu_f(zz.w);
    reinterpret_cast<float4*>(out + wid * kHd)[lane] = o;
}

}  // namespace

size_t dn_prefill_ws_bytes(int batch, int T) {
    // fp16 hi+lo planes: q,k (16 heads each) and v (32 heads); f32 g, beta
    return (size_t)batch * T * (2 * kNumQK + kNumV) * kHd * 2 * 2 + (size_t)batch * kNumV * T * 8 + 1024;
}

cudaError_t launch_dn_prefill(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                              const uint16_t* qkv, const float* a, const float* bgate, float* y,
                              const float* z, float* out) {
    const int B = st->batch;
    cudaStream_t s = ctx->stream;
    const size_t nq = (size_t)B * kNumQK * T * kHd, nv = (size_t)B * kNumV * T * kHd;
    uint16_t* qh = static_cast<uint16_t*>(ctx->ws);
    uint16_t* ql = qh + nq;
    uint16_t* kh = ql + nq;
    uint16_t* kl = kh + nq;
    uint16_t* vh = kl + nq;
    uint16_t* vl = vh + nv;
    float* g = reinterpret_cast<float*>(vl + nv);
    float* be = g + (size_t)B * kNumV * T;
    {
        TimedLaunch tl(ctx, "dn_prefill_prep");
        dim3 grid((T + kPrepTok - 1) / kPrepTok, 2 * kNumQK + kNumV, B);
        dn_prefill_prep<<<grid, 128, 0, s>>>(qkv, a, bgate, p->conv_w, p->a_log, p->dt_bias, st->conv,
                                             st->conv_pos, T, qh, ql, kh, kl, vh, vl, g, be);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    dn_conv_ring<<<dim3(kQKVDim / 256, B), 256, 0, s>>>(qkv, st->conv, st->conv_pos, T);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    CUtensorMap m[6];
    uint16_t* planes[6] = {qh, ql, kh, kl, vh, vl};
    for (int i = 0; i < 6; i++) {
        const uint64_t np = (uint64_t)B * (i < 4 ? kNumQK : kNumV);
        if (encode_rows_tmap(&m[i], planes[i], kHd, (uint64_t)T, np, 64, 64, true) != QM_OK)
            return cudaErrorInvalidValue;
    }
    static bool attr_set[64] = {};
    if (ctx->device < 64 && !attr_set[ctx->device]) {
        e = cudaFuncSetAttribute(dn_prefill_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize, kChunkSmem);
        if (e != cudaSuccess) return e;
        attr_set[ctx->device] = true;
    }
    float* yy = y;  // the gate reads the raw y
    {
        TimedLaunch tl(ctx, "dn_prefill_chunk");
        dn_prefill_chunk<<<dim3(kNumV, B), 128, kChunkSmem, s>>>(m[0], m[1], m[2], m[3], m[4], m[5], g,
                                                                  be, st->s, yy, T, ctx->d_err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    if (z) {
        const size_t nh = (size_t)B * T * kNumV;
        dn_prefill_gate<<<(unsigned)((nh + 7) / 8), 256, 0, s>>>(yy, z, p->norm_gamma, out, nh);
        e = cudaGetLastError();
        if (e == cudaSuccess) ctx->launches += 1;
    }
    return e;
}

}  // namespace qm

using namespace qm;

extern "C" int qm_dn_prefill(qm_ctx* c, const qm_dn_params* p, qm_dn_state* st, int T,
                             const uint16_t* qkv, const float* a, const float* b, float* y,
                             const float* z, float* out) {
    if (!c) return QM_E_ARG;
    if (!p || !p->conv_w || !p->a_log || !p->dt_bias || (z && !p->norm_gamma))
        return set_error(c, QM_E_ARG, "DeltaNet params: null pointer");
    if (!st || !qkv || !a || !b || !y || T <= 0 || (out && !z) || (z && !out))
        return set_error(c, QM_E_ARG, "qm_dn_prefill: null pointer, T <= 0, or out without z");
    if (st->ctx != c) return set_error(c, QM_E_MISMATCH, "state belongs to another context");
    if (st->nvh != kNumV)
        return set_error(c, QM_E_UNSUPPORTED, "qm_dn_prefill: head-sharded states are decode-only");
    if ((uintptr_t)p->conv_w & 15) return set_error(c, QM_E_ARG, "conv_w must be 16-byte aligned");
    if ((y && ((uintptr_t)y & 15)) || (out && ((uintptr_t)out & 15)) || (z && ((uintptr_t)z & 15)))
        return set_error(c, QM_E_ARG, "qm_dn_prefill: y/z/out must be 16-byte aligned");
    cudaSetDevice(c->device);
    int rc = ensure_workspace(c, dn_prefill_ws_bytes(st->batch, T));
    if (rc) return rc;
    cudaError_t e = launch_dn_prefill(c, p, st, T, qkv, a, b, y, z, out);
    if (e != cudaSuccess) return cuda_error(c, e, "dn_prefill launch");
    st->conv_pos += T;
    return QM_OK;
}
