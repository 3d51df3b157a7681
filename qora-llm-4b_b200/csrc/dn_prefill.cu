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
// prep: one warp per (head-vector, run of 16 tokens, sequence); lane l owns
// the 4 channels 4l..4l+3 of the 128-channel head-vector (8-byte bf16 loads,
// the conv history of those channels kept in registers along the run).
// head-vectors 0..15 = q heads, 16..31 = k heads, 32..63 = v heads
// ---------------------------------------------------------------------------
constexpr int kPrepRun = 16;
constexpr int kPrepWarps = 4;  // warps per CTA

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// SiLU with an approximate division (2 ulp): the prep kernel writes its
// activations as fp16 hi + lo (22 significant bits), well above that error,
// and the IEEE division's multi-instruction sequence was a third of its
// special-function-unit work.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float4 bf16x4_to_f32(uint2 u) {
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

__global__ void __launch_bounds__(32 * kPrepWarps)
dn_prefill_prep(const uint16_t* __restrict__ qkv, const float* __restrict__ a_in,
                const float* __restrict__ b_in, const float* __restrict__ conv_w,
                const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                const float* __restrict__ ring, int64_t conv_pos, int T, int nruns,
                uint16_t* __restrict__ qh, uint16_t* __restrict__ ql, uint16_t* __restrict__ kh,
                uint16_t* __restrict__ kl, uint16_t* __restrict__ vh, uint16_t* __restrict__ vl,
                float* __restrict__ gout, float* __restrict__ bout, int B, int* err) {
    const int lane = threadIdx.x & 31;
    const size_t gw = (size_t)blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
    const int hv = (int)(gw % 64);  // adjacent warps read adjacent 256-byte slices of a token row
    const size_t rest = gw / 64;
    const int run = (int)(rest % nruns);
    const int b = (int)(rest / nruns);
    if (b >= B) return;
    const int t0 = run * kPrepRun;
    const int ch = hv * kHd + lane * 4;  // first of this lane's 4 channels
    float4 w[4];                          // w[c] = taps of channel ch + c
#pragma unroll
    for (int c = 0; c < 4; c++) w[c] = reinterpret_cast<const float4*>(conv_w)[ch + c];
    const uint16_t* xb = qkv + (size_t)b * T * kQKVDim + ch;
    const float* rb = ring + (size_t)b * kConvSlots * kQKVDim + ch;
    auto xval = [&](int t) -> float4 {  // raw inputs of token t (negative: the history ring)
        if (t >= 0) return bf16x4_to_f32(*reinterpret_cast<const uint2*>(xb + (size_t)t * kQKVDim));
        const int64_t tok = conv_pos + t;
        if (tok < 0) return make_float4(0.f, 0.f, 0.f, 0.f);
        return *reinterpret_cast<const float4*>(rb + (size_t)(tok & 3) * kQKVDim);
    };
    float4 x3 = xval(t0 - 3), x2 = xval(t0 - 2), x1 = xval(t0 - 1);
    const bool is_q = hv < kNumQK, is_qk = hv < 2 * kNumQK;
    uint16_t *ph, *pl;
    size_t plane;
    if (is_q) {
        ph = qh; pl = ql; plane = (size_t)b * kNumQK + hv;
    } else if (is_qk) {
        ph = kh; pl = kl; plane = (size_t)b * kNumQK + (hv - kNumQK);
    } else {
        ph = vh; pl = vl; plane = (size_t)b * kNumV + (hv - 2 * kNumQK);
    }
    const int tend = min(kPrepRun, T - t0);
    uint2 raw[kPrepRun];  // the run's raw inputs, all loads in flight at once
#pragma unroll
    for (int i = 0; i < kPrepRun; i++)
        raw[i] = (i < tend) ? *reinterpret_cast<const uint2*>(xb + (size_t)(t0 + i) * kQKVDim)
                            : make_uint2(0u, 0u);
#pragma unroll
    for (int i = 0; i < kPrepRun; i++) {
        if (i >= tend) break;
        const float4 x0 = bf16x4_to_f32(raw[i]);
        // gemv.rs:1134-1139: history oldest first, then the token itself
        float a[4];
        const float* h3 = &x3.x;
        const float* h2 = &x2.x;
        const float* h1 = &x1.x;
        const float* h0 = &x0.x;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float cv = h3[c] * w[c].x;
            cv += h2[c] * w[c].y;
            cv += h1[c] * w[c].z;
            cv += h0[c] * w[c].w;
            a[c] = silu_fast(cv);
        }
        x3 = x2;
        x2 = x1;
        x1 = x0;
        if (is_qk) {  // l2_normalize (gemv.rs:641-649, 1153-1155), q * 1/sqrt(128)
            float ss = a[0] * a[0] + a[1] * a[1] + a[2] * a[2] + a[3] * a[3];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float n = sqrtf(ss);
            const float inv = n > 1e-12f ? 1.0f / n : 1.0f;
            const float sc = is_q ? 0.08838834764831845f : 1.0f;
#pragma unroll
            for (int c = 0; c < 4; c++) a[c] = (a[c] * inv) * sc;
        }
        const __half2 h01 = __floats2half2_rn(a[0], a[1]), h23 = __floats2half2_rn(a[2], a[3]);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(a[0] - f01.x, a[1] - f01.y);
        const __half2 l23 = __floats2half2_rn(a[2] - f23.x, a[3] - f23.y);
        const size_t o = (plane * T + t0 + i) * kHd + lane * 4;
        if (!QM_IN(o, 4, (size_t)B * (is_qk ? kNumQK : kNumV) * T * kHd, err)) continue;
        *reinterpret_cast<uint2*>(ph + o) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
        *reinterpret_cast<uint2*>(pl + o) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
    }
    if (!is_qk && lane < tend) {
        // gates of V head vhh for token t0 + lane (gemv.rs:1171-1172), as log-decay
        const int vhh = hv - 2 * kNumQK, t = t0 + lane;
        if (!QM_IN(((size_t)b * kNumV + vhh) * T + t, 1, (size_t)B * kNumV * T, err)) return;
        const float x = a_in[((size_t)b * T + t) * kNumV + vhh] + dt_bias[vhh];
        const float sp = x > 20.0f ? x : log1pf(__expf(x));
        gout[((size_t)b * kNumV + vhh) * T + t] = -__expf(a_log[vhh]) * sp;
        bout[((size_t)b * kNumV + vhh) * T + t] =
            1.0f / (1.0f + __expf(-b_in[((size_t)b * T + t) * kNumV + vhh]));
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
// chunk kernels
// ---------------------------------------------------------------------------
constexpr uint32_t kNegA = 1u << 13;
constexpr uint32_t kIdKK = umma_idesc_f16kind(128, 64, false, false, false);   // A K, B K
constexpr uint32_t kIdW = umma_idesc_f16kind(128, 64, true, false, false);     // A MN, B K
constexpr uint32_t kIdSW = umma_idesc_f16kind(128, 64, false, true, false) | kNegA;  // -A . B(MN)
constexpr uint32_t kIdSQ = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUP = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUK = umma_idesc_f16kind(128, 128, false, true, false);   // A K, B MN

__device__ __forceinline__ uint32_t h2bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// two f32 -> fp16 hi pair and the fp16 of the remainders (packed conversions)
__device__ __forceinline__ void split2(float a, float b, __half2& hi, __half2& lo) {
    hi = __floats2half2_rn(a, b);
    const float2 f = __half22float2(hi);
    lo = __floats2half2_rn(a - f.x, b - f.y);
}

// 8 consecutive f32 -> fp16 hi (and lo = fp16 of the remainder) as two uint4
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        __half2 a, b;
        split2(v[2 * i], v[2 * i + 1], a, b);
        h[i] = h2bits(a);
        l[i] = h2bits(b);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ uint4 round8(const float* v) {
    return make_uint4(pack_f16x2_rn(v[0], v[1]), pack_f16x2_rn(v[2], v[3]),
                      pack_f16x2_rn(v[4], v[5]), pack_f16x2_rn(v[6], v[7]));
}

// inclusive cumulative log-decay of the 64 gates in sg[] (warp 0), in log2
// units: sG[t] = log2e * G_t; plus eG[t] = e^G_t and eD[s] = e^(G_63 - G_s)
__device__ __forceinline__ void chunk_decays(const float* sg, float* sG, float* eG, float* eD,
                                             int lane) {
    float g0 = sg[lane] * kLog2e, g1 = sg[lane + 32] * kLog2e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u0 = __shfl_up_sync(0xffffffffu, g0, o);
        const float u1 = __shfl_up_sync(0xffffffffu, g1, o);
        if (lane >= o) {
            g0 += u0;
            g1 += u1;
        }
    }
    g1 += __shfl_sync(0xffffffffu, g0, 31);
    const float g63 = __shfl_sync(0xffffffffu, g1, 31);
    sG[lane] = g0;
    sG[lane + 32] = g1;
    if (eG) {
        eG[lane] = exp2f(g0);
        eG[lane + 32] = exp2f(g1);
        eD[lane] = exp2f(g63 - g0);
        eD[lane + 32] = exp2f(g63 - g1);
    }
}

// One block diagonal d (pairs (i, j) = (j + d, j), j = 0 .. 3-d) of the blocked
// unit-lower-triangular inverse T of I + A (row stride kAStride floats):
//   X_ij = sum_{k=j}^{i-1} A_ik T_kj   (kept in the unused upper block (j, i))
//   T_ij = -T_ii X_ij                  (T_ii stored with zeros above its diagonal)
// Each of the NT threads owns (4 - d) * 256 / NT elements; all trip counts
// are compile-time so the shared-memory loads issue ahead of the FMAs.
template <int D, int NT>
__device__ __forceinline__ void tri_inverse_diagonal(const float* __restrict__ A, float* __restrict__ Tm,
                                                     int tid) {
    constexpr int kStride = 68;
    constexpr int NOUT = (4 - D) * 256 / NT;
#pragma unroll
    for (int m = 0; m < NOUT; m++) {
        const int o = tid + NT * m;
        const int j = o >> 8, i = j + D, r = (o >> 4) & 15, c = o & 15;
        const float* arow = A + (16 * i + r) * kStride + 16 * j;
        const float* tcol = Tm + (16 * j) * kStride + 16 * j + c;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 16 * D; u += 4) {
            const float4 a = *reinterpret_cast<const float4*>(arow + u);
            x[0] = fmaf(a.x, tcol[(u + 0) * kStride], x[0]);
            x[1] = fmaf(a.y, tcol[(u + 1) * kStride], x[1]);
            x[2] = fmaf(a.z, tcol[(u + 2) * kStride], x[2]);
            x[3] = fmaf(a.w, tcol[(u + 3) * kStride], x[3]);
        }
        Tm[(16 * j + r) * kStride + 16 * i + c] = (x[0] + x[1]) + (x[2] + x[3]);
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < NOUT; m++) {
        const int o = tid + NT * m;
        const int j = o >> 8, i = j + D, r = (o >> 4) & 15, c = o & 15;
        const float* trow = Tm + (16 * i + r) * kStride + 16 * i;
        const float* xcol = Tm + (16 * j) * kStride + 16 * i + c;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < 16; u += 4) {
            const float4 t = *reinterpret_cast<const float4*>(trow + u);
            x[0] = fmaf(t.x, xcol[(u + 0) * kStride], x[0]);
            x[1] = fmaf(t.y, xcol[(u + 1) * kStride], x[1]);
            x[2] = fmaf(t.z, xcol[(u + 2) * kStride], x[2]);
            x[3] = fmaf(t.w, xcol[(u + 3) * kStride], x[3]);
        }
        Tm[(16 * i + r) * kStride + 16 * j + c] = -((x[0] + x[1]) + (x[2] + x[3]));
    }
    __syncthreads();
}

struct ChunkBars {
    uint64_t load, mma;
    uint32_t tmem_base;
    int abort_flag;
};

// ---- 2a. chunk-local WY factors: one CTA (8 warps) per (V head, chunk, sequence) ----
//
// Everything in a chunk that does not depend on the state entering it:
//   MMA1  [K;Q] K^T                       (compensated)  -> A (f32) and P'
//   T = (I + A)^-1 by forward substitution, one column per thread (f32)
//   MMA2  W^T  = K^T (T diag(b e^G))^T    (compensated)
//   MMA3  U~^T = V^T (T diag(b))^T        (compensated)
// written to the workspace for the state pass: W^T fp16 [128 k][64 t],
// U~^T f32 as [16][128 v][4] (float4 of 4 tokens per v, so the state pass
// loads it with one bulk copy and reads it conflict-free), P' fp16 hi/lo
// [64 t][64 s], and the decayed operands of the state products
// Q~_t = e^G_t q_t (fp16) and K~_s = e^(G_63 - G_s) k_s (fp16 hi/lo), [64][128].
// 102 KB of shared memory and 256 TMEM columns: two CTAs per SM.  Warps w and
// w+4 share TMEM lane quarter w%4 and split the 64 columns of every TMEM tile.
constexpr int kL_KQh = 0;              // [K;Q] hi: 2 boxes [128 rows x 64] fp16 (K rows 0-63,
constexpr int kL_KQl = 32768;          //   Q rows 64-127); after MMA1 the four Q quarters
constexpr int kL_T1h = kL_KQh + 8192;  //   hold T' and T'' (hi/lo), 8 KB each
constexpr int kL_T1l = kL_KQh + 24576;
constexpr int kL_T2h = kL_KQl + 8192;
constexpr int kL_T2l = kL_KQl + 24576;
constexpr int kAStride = 68;           // floats per A / T row (float4-aligned)
constexpr int kL_A = 65536;            // A f32 [64][68] and T f32 [64][68] during the
constexpr int kL_Tm = kL_A + 64 * kAStride * 4;  // solve, then V hi (2 boxes [64 x 64])
constexpr int kL_Vh = 65536;           //   and V lo on top of them
constexpr int kL_Vl = 81920;
constexpr int kL_Misc = kL_Tm + 64 * kAStride * 4;  // G, beta, g, b e^G, e^G, e^(G63-G): 6 x 64 f32
constexpr int kLocalSmem = kL_Misc + 6 * 64 * 4 + 64 + 1024;
static_assert(kL_Vl + 16384 <= kL_Misc, "V fits over A and T");
constexpr uint32_t kTmKQ = 0, kTmW = 64, kTmU = 128;
constexpr int kLocalThreads = 256;

__global__ void __launch_bounds__(kLocalThreads, 2)
dn_chunk_local(const __grid_constant__ CUtensorMap tqh, const __grid_constant__ CUtensorMap tql,
               const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
               const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
               const float* __restrict__ gin, const float* __restrict__ bin, int T, int nch,
               uint16_t* __restrict__ wt_out, float* __restrict__ ut_out,
               uint16_t* __restrict__ ph_out, uint16_t* __restrict__ pl_out,
               uint16_t* __restrict__ qt_out, uint16_t* __restrict__ kth_out,
               uint16_t* __restrict__ ktl_out, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* sG = reinterpret_cast<float*>(smem + kL_Misc);
    float* sB = sG + 64;
    float* sg = sB + 64;
    float* sC1 = sg + 64;  // b_j e^G_j
    float* eG = sC1 + 64;
    float* eD = eG + 64;
    ChunkBars* bars = reinterpret_cast<ChunkBars*>(eD + 64);
    float* Amat = reinterpret_cast<float*>(smem + kL_A);
    float* Tm = reinterpret_cast<float*>(smem + kL_Tm);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sb = smem_u32(smem);

    const int vh = blockIdx.x, ci = blockIdx.y, b = blockIdx.z, qk = vh >> 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;  // TMEM lanes 32*quarter.., columns 32*half..
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int row = quarter * 32 + lane;              // TMEM lane = tile row
    const int t0 = ci * kC, tc = min(kC, T - t0);
    const size_t plane_qk = (size_t)b * kNumQK + qk, plane_v = (size_t)b * kNumV + vh;
    const size_t item = ((size_t)b * kNumV + vh) * nch + ci;

    if (tid == 0) {
        mbar_init(smem_u32(&bars->load), 1);
        mbar_init(smem_u32(&bars->mma), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&bars->tmem_base), 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = bars->tmem_base;

    // thread 0's record of the last phase it started on each barrier and not
    // yet seen complete (drained on the way out of an aborted CTA)
    bool ld_out = false, mm_out = false;
    uint32_t ld_par = 0, mm_par = 0;
    if (tid == 0) {
        const uint32_t lb = smem_u32(&bars->load);
        mbar_arrive_expect_tx(lb, 8 * 8192);
        ld_out = true;
        for (int hb = 0; hb < 2; hb++) {
            tma_load_3d(sb + kL_KQh + hb * 16384, &tkh, hb * 64, t0, (int)plane_qk, lb);
            tma_load_3d(sb + kL_KQl + hb * 16384, &tkl, hb * 64, t0, (int)plane_qk, lb);
            tma_load_3d(sb + kL_KQh + hb * 16384 + 8192, &tqh, hb * 64, t0, (int)plane_qk, lb);
            tma_load_3d(sb + kL_KQl + hb * 16384 + 8192, &tql, hb * 64, t0, (int)plane_qk, lb);
        }
    }
    if (tid < kC) {
        const bool valid = tid < tc;
        sg[tid] = valid ? gin[plane_v * T + t0 + tid] : 0.f;
        sB[tid] = valid ? bin[plane_v * T + t0 + tid] : 0.f;
    }
    __syncthreads();
    if (warp == 0) chunk_decays(sg, sG, eG, eD, lane);
    bool ok = mbar_wait_bounded(smem_u32(&bars->load), 0, abort_flag, err);
    if (ok) ld_out = false;
    ok = __syncthreads_and(ok) != 0;  // also publishes sG

    // ---- MMA1: [K;Q] K^T (compensated) -> TMEM KQ ----
    if (ok && tid == 0) {
        tc_fence_after();
        int n = 0;
        for (int term = 0; term < 3; term++) {
            const uint32_t abase = sb + (term == 2 ? kL_KQl : kL_KQh);
            const uint32_t bbase = sb + (term == 1 ? kL_KQl : kL_KQh);
            for (int kk = 0; kk < 8; kk++, n++) {
                const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                umma_bf16_ss(tm + kTmKQ, umma_sdesc(abase + off, 16, 1024),
                             umma_sdesc(bbase + off, 16, 1024), kIdKK, n > 0);
            }
        }
        umma_commit(smem_u32(&bars->mma));
        mm_out = true;
    }
    if (ok) {
        ok = mbar_wait_bounded(smem_u32(&bars->mma), 0, abort_flag, err);
        if (ok) mm_out = false;
    }
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();

    // ---- rows 0-63: A (f32, shared); rows 64-127: P' hi/lo (global); this
    // thread's 32 columns [s0, s0 + 32) ----
    if (ok) {
        float kq[32];
        const int s0 = half * 32;
        tmem_ld32(tm + lane_addr + kTmKQ + s0, kq);
        tmem_ld_wait();
        if (row < kC) {
            const int t = row;
            const float Gt = sG[t], bt = sB[t];
            float* arow = Amat + t * kAStride + s0;
            if (QM_IN(t * kAStride + s0, 32, kC * kAStride, err))
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const int s = s0 + i;
                float4 v;
                v.x = (s + 0 < t) ? bt * ex2_approx(Gt - sG[s + 0]) * kq[i + 0] : 0.f;
                v.y = (s + 1 < t) ? bt * ex2_approx(Gt - sG[s + 1]) * kq[i + 1] : 0.f;
                v.z = (s + 2 < t) ? bt * ex2_approx(Gt - sG[s + 2]) * kq[i + 2] : 0.f;
                v.w = (s + 3 < t) ? bt * ex2_approx(Gt - sG[s + 3]) * kq[i + 3] : 0.f;
                *reinterpret_cast<float4*>(arow + i) = v;
            }
        } else {
            const int t = row - kC;
            const float Gt = sG[t];
            const size_t items = (size_t)gridDim.x * gridDim.y * gridDim.z;
            if (QM_IN((item * kC + t) * kC + s0, 32, items * kC * kC, err)) {
                uint4* hrow = reinterpret_cast<uint4*>(ph_out + (item * kC + t) * kC + s0);
                uint4* lrow = reinterpret_cast<uint4*>(pl_out + (item * kC + t) * kC + s0);
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    float p[8];
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const int s = s0 + i + q;
                        p[q] = (s <= t) ? ex2_approx(Gt - sG[s]) * kq[i + q] : 0.f;
                    }
                    uint4 h, l;
                    split8(p, h, l);
                    hrow[i / 8] = h;
                    lrow[i / 8] = l;
                }
            }
        }
    }
    // ---- Q~ = e^G q (fp16) and K~ = e^(G63-G) k (fp16 hi/lo), from the hi/lo tiles ----
    if (ok && QM_IN(item * kC * kHd, kC * kHd, (size_t)gridDim.x * gridDim.y * gridDim.z * kC * kHd, err)) {
        const size_t rowbase = item * kC;
#pragma unroll 2
        for (int m = 0; m < 1024 / kLocalThreads; m++) {
            const int o = tid + kLocalThreads * m, t = o >> 4, kc = o & 15;
            const uint32_t off = (kc >> 3) * 16384 + sw128_off(t, kc & 7);
            float v[8];
            // Q rows sit 8 KB into each box
            uint4 h = *reinterpret_cast<const uint4*>(smem + kL_KQh + 8192 + off);
            uint4 l = *reinterpret_cast<const uint4*>(smem + kL_KQl + 8192 + off);
            const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hw[i]));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&lw[i]));
                v[2 * i] = (a.x + b.x) * eG[t];
                v[2 * i + 1] = (a.y + b.y) * eG[t];
            }
            reinterpret_cast<uint4*>(qt_out + (rowbase + t) * kHd)[kc] = round8(v);
            h = *reinterpret_cast<const uint4*>(smem + kL_KQh + off);
            l = *reinterpret_cast<const uint4*>(smem + kL_KQl + off);
            const uint32_t hk[4] = {h.x, h.y, h.z, h.w}, lk[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hk[i]));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&lk[i]));
                v[2 * i] = (a.x + b.x) * eD[t];
                v[2 * i + 1] = (a.y + b.y) * eD[t];
            }
            uint4 kh4, kl4;
            split8(v, kh4, kl4);
            reinterpret_cast<uint4*>(kth_out + (rowbase + t) * kHd)[kc] = kh4;
            reinterpret_cast<uint4*>(ktl_out + (rowbase + t) * kHd)[kc] = kl4;
        }
    }
    tc_fence_before();
    __syncthreads();

    // ---- T = (I + A)^-1, blocked by 16: diagonal blocks by forward substitution,
    // then T_ij = -T_ii sum_{k=j}^{i-1} A_ik T_kj by block diagonals i - j = 1, 2, 3
    // (f32); the upper blocks of T's storage hold the partial sums X_ij ----
    if (ok) {  // block-uniform
        if (tid < kC) {
            const int blk = tid >> 4, c = tid & 15, o = blk * 16;
            float tc[16];
#pragma unroll
            for (int r = 0; r < 16; r++) {
                const float* arow = Amat + (o + r) * kAStride + o;
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int u = 0; u + 1 < r; u += 2) {
                    a0 = fmaf(arow[u], tc[u], a0);
                    a1 = fmaf(arow[u + 1], tc[u + 1], a1);
                }
                if (r & 1) a0 = fmaf(arow[r - 1], tc[r - 1], a0);
                tc[r] = (r == c) ? 1.f : (r < c ? 0.f : -(a0 + a1));
            }
#pragma unroll
            for (int r = 0; r < 16; r++) Tm[(o + r) * kAStride + o + c] = tc[r];
        } else if (tid < 2 * kC) {
            const int t = tid - kC;
            sC1[t] = sB[t] * eG[t];
        }
        __syncthreads();
        static_assert(kAStride == 68, "tri_inverse_diagonal assumes the A/T row stride");
        tri_inverse_diagonal<1, kLocalThreads>(Amat, Tm, tid);
        tri_inverse_diagonal<2, kLocalThreads>(Amat, Tm, tid);
        tri_inverse_diagonal<3, kLocalThreads>(Amat, Tm, tid);
        // T' = T diag(b e^G), T'' = T diag(b) as fp16 hi/lo [t][j] tiles (upper part zero)
        for (int o = tid; o < kC * 8; o += kLocalThreads) {
            const int t = o >> 3, jc = o & 7, j0 = jc * 8;
            float v1[8], v2[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const int j = j0 + q;
                const float tv = (j <= t) ? Tm[t * kAStride + j] : 0.f;
                v1[q] = tv * sC1[j];
                v2[q] = tv * sB[j];
            }
            uint4 h, l;
            split8(v1, h, l);
            *reinterpret_cast<uint4*>(smem + kL_T1h + sw128_off(t, jc)) = h;
            *reinterpret_cast<uint4*>(smem + kL_T1l + sw128_off(t, jc)) = l;
            split8(v2, h, l);
            *reinterpret_cast<uint4*>(smem + kL_T2h + sw128_off(t, jc)) = h;
            *reinterpret_cast<uint4*>(smem + kL_T2l + sw128_off(t, jc)) = l;
        }
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();  // A is dead from here: V lands on it

    // ---- MMA2 (W^T) now; V load; MMA3 (U~^T) once V has landed ----
    if (ok && tid == 0) {
        const uint32_t lb = smem_u32(&bars->load);
        mbar_arrive_expect_tx(lb, 4 * 8192);
        ld_out = true;
        ld_par = 1;
        for (int hb = 0; hb < 2; hb++) {
            tma_load_3d(sb + kL_Vh + hb * 8192, &tvh, hb * 64, t0, (int)plane_v, lb);
            tma_load_3d(sb + kL_Vl + hb * 8192, &tvl, hb * 64, t0, (int)plane_v, lb);
        }
        tc_fence_after();
        int n = 0;
        for (int term = 0; term < 3; term++) {
            const uint32_t ka = sb + (term == 2 ? kL_KQl : kL_KQh);
            const uint32_t tb = sb + (term == 1 ? kL_T1l : kL_T1h);
            for (int kk = 0; kk < 4; kk++, n++)
                umma_bf16_ss(tm + kTmW, umma_sdesc(ka + kk * 2048, 16384, 1024),
                             umma_sdesc(tb + kk * 32, 16, 1024), kIdW, n > 0);
        }
        if (mbar_wait_bounded(lb, 1, abort_flag, err)) {
            ld_out = false;
            tc_fence_after();
            n = 0;
            for (int term = 0; term < 3; term++) {
                const uint32_t va = sb + (term == 2 ? kL_Vl : kL_Vh);
                const uint32_t tb = sb + (term == 1 ? kL_T2l : kL_T2h);
                for (int kk = 0; kk < 4; kk++, n++)
                    umma_bf16_ss(tm + kTmU, umma_sdesc(va + kk * 2048, 8192, 1024),
                                 umma_sdesc(tb + kk * 32, 16, 1024), kIdW, n > 0);
            }
        }
        umma_commit(smem_u32(&bars->mma));  // also covers MMA2 when the V wait gave up
        mm_out = true;
        mm_par = 1;
    }
    if (ok) {
        ok = mbar_wait_bounded(smem_u32(&bars->mma), 1, abort_flag, err);
        if (ok) mm_out = false;
    }
    ok = __syncthreads_and(ok && !*abort_flag) != 0;
    tc_fence_after();

    // ---- outputs: W^T row k (fp16), U~^T row v (f32, [t/4][v][4]); this
    // thread's 32 tokens [32 half, 32 half + 32) ----
    if (ok && QM_IN(item * kHd * kC, kHd * kC, (size_t)gridDim.x * gridDim.y * gridDim.z * kHd * kC, err)) {
        float wv[32];
        tmem_ld32(tm + lane_addr + kTmW + half * 32, wv);
        tmem_ld_wait();
        uint4* wrow = reinterpret_cast<uint4*>(wt_out + (item * kHd + row) * kC) + half * 4;
#pragma unroll
        for (int t = 0; t < 32; t += 8) wrow[t / 8] = round8(wv + t);
        float uv[32];
        tmem_ld32(tm + lane_addr + kTmU + half * 32, uv);
        tmem_ld_wait();
        float4* ub = reinterpret_cast<float4*>(ut_out + item * kHd * kC);
#pragma unroll
        for (int i = 0; i < 8; i++)
            ub[(half * 8 + i) * kHd + row] = make_float4(uv[4 * i], uv[4 * i + 1], uv[4 * i + 2], uv[4 * i + 3]);
    }
    if (tid == 0) {
        if (ld_out) mbar_drain(smem_u32(&bars->load), ld_par);
        if (mm_out) mbar_drain(smem_u32(&bars->mma), mm_par);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, 256);
    }
}

// ---- 2b. state pass: one CTA (128 threads, lane = v row) per (V head, sequence) ----
//
// Per chunk c, with S0 the state entering it (f32 master in TMEM, fp16 copy in
// shared memory as the A operand), Q~ = e^G Q and K~ = e^(G63-G) K:
//   MMA4  U_acc = -S0 W^T                    MMA5  Y[c&1] = S0 Q~^T  (fp16)
//   U = U~ + U_acc (f32) -> fp16 hi/lo
//   MMA7  dS = U^T K~   (compensated)        MMA6  Y[c&1] += U^T P'^T (compensated)
//   S_master = e^G63 S_master + dS (f32), and its fp16 copy for chunk c+1
// The dependency chain per chunk is S copy -> MMA4 -> U -> MMA7 -> S copy;
// MMA5, MMA6 and the output of chunk c-1 (y = Y[(c-1)&1], read while MMA7
// runs) stay off it.  W^T, Q~ and U~ (one untiled bulk copy) are refetched
// for chunk c+1 as soon as MMA4/MMA5 and the U step are done, K~ after MMA7,
// and P' is double-buffered; the gates of chunk c+1 are read into registers
// during chunk c.
constexpr int kS_S0 = 0;            // S0 fp16 [128 v x 128 k]: 2 boxes [128 x 64]
constexpr int kS_W = 32768;         // W^T [128 k x 64 t] fp16 (16 KB)
constexpr int kS_Q = 49152;         // Q~ [64 t x 128 k] fp16: 2 boxes [64 x 64] (16 KB)
constexpr int kS_Ut = 65536;        // U~^T f32 [16][128 v][4] (32 KB)
constexpr int kS_P = 98304;         // P' hi, lo [64 t x 64 s] (8 KB each), x2 buffers (32 KB)
constexpr int kS_Kh = 131072;       // K~ hi [64 s x 128 k]: 2 boxes [64 x 64]
constexpr int kS_Kl = 147456;
constexpr int kS_Uh = 163840;       // U^T hi [128 v x 64 s]
constexpr int kS_Ul = 180224;
constexpr int kS_Misc = 196608;     // [2] x (G, eG, eD, g): 8 x 64 f32; barriers
constexpr int kStateSmem = kS_Misc + 8 * 64 * 4 + 128 + 1024;
constexpr uint32_t kTmU2 = 0, kTmY = 64 /* x2 */, kTmDS = 256, kTmS = 384;

struct StateBars {
    uint64_t wqu_full, k_full, p_full[2], m4, m5, m7, mY;
    uint32_t tmem_base;
    int abort_flag;
};

__global__ void __launch_bounds__(128, 1)
dn_chunk_state(const __grid_constant__ CUtensorMap twt, const __grid_constant__ CUtensorMap tph,
               const __grid_constant__ CUtensorMap tpl, const __grid_constant__ CUtensorMap tqt,
               const __grid_constant__ CUtensorMap tkth, const __grid_constant__ CUtensorMap tktl,
               const float* __restrict__ ut_in, const float* __restrict__ gin,
               float* __restrict__ S, float* __restrict__ y, int T, int nch, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* misc = reinterpret_cast<float*>(smem + kS_Misc);
    // per chunk parity p: sG = misc + p*256, eG = +64, eD = +128, sg = +192
    StateBars* bars = reinterpret_cast<StateBars*>(misc + 8 * 64);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sb = smem_u32(smem);

    const int vh = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
    const int row = tid;  // TMEM lane = v row
    const size_t plane_v = (size_t)b * kNumV + vh;
    const size_t item0 = plane_v * nch;

    if (tid == 0) {
        mbar_init(smem_u32(&bars->wqu_full), 1);
        mbar_init(smem_u32(&bars->k_full), 1);
        mbar_init(smem_u32(&bars->p_full[0]), 1);
        mbar_init(smem_u32(&bars->p_full[1]), 1);
        mbar_init(smem_u32(&bars->m4), 1);
        mbar_init(smem_u32(&bars->m5), 1);
        mbar_init(smem_u32(&bars->m7), 1);
        mbar_init(smem_u32(&bars->mY), 1);
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

    // thread 0's record of the last phase it started on each barrier and not
    // yet seen complete (drained on the way out of an aborted CTA)
    bool out_[8] = {false, false, false, false, false, false, false, false};
    uint32_t par_[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint64_t* const bar_list[8] = {&bars->wqu_full, &bars->k_full, &bars->p_full[0], &bars->p_full[1],
                                   &bars->m4, &bars->m5, &bars->m7, &bars->mY};
    auto started = [&](int i, int c) { out_[i] = true; par_[i] = (uint32_t)c & 1; };
    auto seen = [&](int i) { out_[i] = false; };
    enum { kWqu = 0, kK = 1, kP0 = 2, kM4 = 4, kM5 = 5, kM7 = 6, kMY = 7 };

    auto issue_wqu = [&](int c) {  // W^T, Q~ and U~^T of chunk c
        const uint32_t fb = smem_u32(&bars->wqu_full);
        started(kWqu, c);
        mbar_arrive_expect_tx(fb, 16384 + 16384 + 32768);
        tma_load_3d(sb + kS_W, &twt, 0, 0, (int)(item0 + c), fb);
        for (int hb = 0; hb < 2; hb++)
            tma_load_3d(sb + kS_Q + hb * 8192, &tqt, hb * 64, 0, (int)(item0 + c), fb);
        if (QM_IN((item0 + c) * kHd * kC, kHd * kC, (size_t)gridDim.x * gridDim.y * nch * kHd * kC, err))
            bulk_load(sb + kS_Ut, ut_in + (item0 + c) * kHd * kC, 32768, fb);
    };
    auto issue_k = [&](int c) {  // K~ hi/lo of chunk c
        const uint32_t fb = smem_u32(&bars->k_full);
        started(kK, c);
        mbar_arrive_expect_tx(fb, 16384 * 2);
        for (int hb = 0; hb < 2; hb++) {
            tma_load_3d(sb + kS_Kh + hb * 8192, &tkth, hb * 64, 0, (int)(item0 + c), fb);
            tma_load_3d(sb + kS_Kl + hb * 8192, &tktl, hb * 64, 0, (int)(item0 + c), fb);
        }
    };
    auto issue_p = [&](int c) {  // P' hi/lo of chunk c into buffer c & 1
        const int buf = c & 1;
        const uint32_t fb = smem_u32(&bars->p_full[buf]);
        started(kP0 + buf, c >> 1);
        mbar_arrive_expect_tx(fb, 8192 * 2);
        tma_load_3d(sb + kS_P + buf * 16384, &tph, 0, 0, (int)(item0 + c), fb);
        tma_load_3d(sb + kS_P + buf * 16384 + 8192, &tpl, 0, 0, (int)(item0 + c), fb);
    };
    if (tid == 0) {
        issue_wqu(0);
        issue_k(0);
        issue_p(0);
        if (nch > 1) issue_p(1);
    }
    float g_next = (tid < min(kC, T)) ? gin[plane_v * T + tid] : 0.f;  // gates of chunk 0

    // ---- initial state: global f32 -> TMEM master and fp16 copy ----
    float* Sg = S + (QM_IN(plane_v * kHd * kHd, kHd * kHd, (size_t)gridDim.x * gridDim.y * kHd * kHd, err)
                         ? plane_v * kHd * kHd : 0);
    {
        const float* srow = Sg + (size_t)row * kHd;
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 f = *reinterpret_cast<const float4*>(srow + c * 32 + i);
                v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
            }
            tmem_st32(tm + lane_addr + kTmS + c * 32, v);
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                const int k = c * 32 + i;
                *reinterpret_cast<uint4*>(smem + kS_S0 + (k >> 6) * 16384 + sw128_off(row, (k & 63) >> 3)) =
                    round8(v + i);
            }
        }
        tmem_st_wait();
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();

    // y of chunk c from Y[c&1] (lane v, coalesced per token); the caller has
    // seen MMA6 of chunk c complete
    auto write_y = [&](int c) {
        const int t0 = c * kC, tc = min(kC, T - t0);
        float yv[64];
        tmem_ld32(tm + lane_addr + kTmY + (c & 1) * 64, yv);
        tmem_ld32(tm + lane_addr + kTmY + (c & 1) * 64 + 32, yv + 32);
        tmem_ld_wait();
        float* yb = y + ((size_t)b * T + t0) * kVDim + (size_t)vh * kHd + row;
        if (!QM_IN(((size_t)b * T + t0 + tc - 1) * kVDim + (size_t)vh * kHd + row, 1,
                   (size_t)gridDim.y * T * kVDim, err))
            return;
#pragma unroll
        for (int t = 0; t < kC; t++)
            if (t < tc) yb[(size_t)t * kVDim] = yv[t];
    };

    bool ok = true;
    for (int ci = 0; ci < nch && ok; ci++) {
        const int p = ci & 1;
        float* sGp = misc + p * 256;
        float* eGp = sGp + 64;
        float* eDp = sGp + 128;
        float* sgp = sGp + 192;
        if (tid < kC) sgp[tid] = g_next;
        {  // gates of chunk ci+1, consumed next iteration
            const int tn = (ci + 1) * kC;
            g_next = (ci + 1 < nch && tid < min(kC, T - tn)) ? gin[plane_v * T + tn + tid] : 0.f;
        }
        __syncthreads();
        if (warp == 0) chunk_decays(sgp, sGp, eGp, eDp, lane);

        // ---- MMA4 (commit m4), MMA5 (commit m5) ----
        if (tid == 0) {
            if (mbar_wait_bounded(smem_u32(&bars->wqu_full), p, abort_flag, err)) {
                seen(kWqu);
                tc_fence_after();
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16_ss(tm + kTmU2, umma_sdesc(sb + kS_S0 + aoff, 16, 1024),
                                 umma_sdesc(sb + kS_W + kk * 2048, 8192, 1024), kIdSW, kk > 0);
                }
                umma_commit(smem_u32(&bars->m4));
                started(kM4, ci);
                for (int kk = 0; kk < 8; kk++) {
                    const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_bf16_ss(tm + kTmY + p * 64, umma_sdesc(sb + kS_S0 + aoff, 16, 1024),
                                 umma_sdesc(sb + kS_Q + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                                 kIdSQ, kk > 0);
                }
            } else {
                umma_commit(smem_u32(&bars->m4));
                started(kM4, ci);
            }
            umma_commit(smem_u32(&bars->m5));
            started(kM5, ci);
        }
        {
            // every thread waits on the load barrier too: it reads U~ from shared memory
            const bool w = mbar_wait_bounded(smem_u32(&bars->m4), p, abort_flag, err) &&
                           mbar_wait_bounded(smem_u32(&bars->wqu_full), p, abort_flag, err);
            if (w) seen(kM4);
            ok = __syncthreads_and(ok && w && !*abort_flag) != 0;  // also publishes G, eG, eD
        }
        if (!ok) break;
        tc_fence_after();
        // MMA6 of chunk ci-1 read P' buffer (ci+1)&1 and finished before MMA4 of ci
        if (tid == 0 && ci + 1 < nch && ci >= 1) issue_p(ci + 1);

        // ---- U = U~ + U_acc -> fp16 hi/lo ----
        {
            float acc[64];
            tmem_ld32(tm + lane_addr + kTmU2, acc);
            tmem_ld32(tm + lane_addr + kTmU2 + 32, acc + 32);
            const float4* ub = reinterpret_cast<const float4*>(smem + kS_Ut);
            float ut[64];
#pragma unroll
            for (int t4 = 0; t4 < kC / 4; t4++) {
                const float4 f = ub[t4 * kHd + row];
                ut[4 * t4] = f.x; ut[4 * t4 + 1] = f.y; ut[4 * t4 + 2] = f.z; ut[4 * t4 + 3] = f.w;
            }
            tmem_ld_wait();
#pragma unroll
            for (int s = 0; s < kC; s += 8) {
                float u8[8];
#pragma unroll
                for (int i = 0; i < 8; i++) u8[i] = acc[s + i] + ut[s + i];
                uint4 h, l;
                split8(u8, h, l);
                *reinterpret_cast<uint4*>(smem + kS_Uh + sw128_off(row, s >> 3)) = h;
                *reinterpret_cast<uint4*>(smem + kS_Ul + sw128_off(row, s >> 3)) = l;
            }
        }
        if (tid == 0) {  // MMA5 must be done before W/Q~ are refilled and S0 is rewritten
            if (mbar_wait_bounded(smem_u32(&bars->m5), p, abort_flag, err)) seen(kM5);
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();

        // ---- MMA7 (commit m7), MMA6 (commit mY); refetch W^T, Q~, U~ for chunk ci+1 ----
        if (tid == 0) {
            if (ci + 1 < nch && !*abort_flag) issue_wqu(ci + 1);
            const bool kok = mbar_wait_bounded(smem_u32(&bars->k_full), p, abort_flag, err);
            const bool pok = kok && mbar_wait_bounded(smem_u32(&bars->p_full[p]), (ci >> 1) & 1, abort_flag, err);
            if (kok) seen(kK);
            if (pok) seen(kP0 + p);
            tc_fence_after();
            if (kok) {
                int n = 0;
                for (int term = 0; term < 3; term++) {
                    const uint32_t ua = sb + (term == 2 ? kS_Ul : kS_Uh);
                    const uint32_t kb = sb + (term == 1 ? kS_Kl : kS_Kh);
                    for (int kk = 0; kk < 4; kk++, n++)
                        umma_bf16_ss(tm + kTmDS, umma_sdesc(ua + kk * 32, 16, 1024),
                                     umma_sdesc(kb + kk * 2048, 8192, 1024), kIdUK, n > 0);
                }
            }
            umma_commit(smem_u32(&bars->m7));
            started(kM7, ci);
            if (pok) {
                const uint32_t pb = sb + kS_P + p * 16384;
                for (int term = 0; term < 3; term++) {
                    const uint32_t ua = sb + (term == 2 ? kS_Ul : kS_Uh);
                    const uint32_t pbt = pb + (term == 1 ? 8192 : 0);
                    for (int kk = 0; kk < 4; kk++)
                        umma_bf16_ss(tm + kTmY + p * 64, umma_sdesc(ua + kk * 32, 16, 1024),
                                     umma_sdesc(pbt + kk * 32, 16, 1024), kIdUP, 1u);
                }
            }
            umma_commit(smem_u32(&bars->mY));
            started(kMY, ci);
        }
        // outputs of chunk ci-1 while MMA7 runs (its MMA6 finished before MMA4 of ci)
        if (ci > 0) write_y(ci - 1);
        {
            const bool w = mbar_wait_bounded(smem_u32(&bars->m7), p, abort_flag, err);
            if (w) seen(kM7);
            ok = __syncthreads_and(ok && w && !*abort_flag) != 0;
        }
        if (!ok) break;
        tc_fence_after();
        if (tid == 0 && ci + 1 < nch) issue_k(ci + 1);  // MMA7 has read K~

        // ---- S_master = e^G63 S_master + dS, and its fp16 copy for the next chunk ----
        const float decay = eGp[kC - 1];
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
            float sv[32], dv[32];
            tmem_ld32(tm + lane_addr + kTmS + c * 32, sv);
            tmem_ld32(tm + lane_addr + kTmDS + c * 32, dv);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) sv[i] = fmaf(sv[i], decay, dv[i]);
            tmem_st32(tm + lane_addr + kTmS + c * 32, sv);
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                const int k = c * 32 + i;
                *reinterpret_cast<uint4*>(smem + kS_S0 + (k >> 6) * 16384 + sw128_off(row, (k & 63) >> 3)) =
                    round8(sv + i);
            }
        }
        tmem_st_wait();
        fence_proxy_async_shared();
        tc_fence_before();
        __syncthreads();
    }

    // ---- outputs of the last chunk; final state back to global (f32) ----
    if (ok) {
        const bool w = mbar_wait_bounded(smem_u32(&bars->mY), (nch - 1) & 1, abort_flag, err);
        if (w) seen(kMY);
        tc_fence_after();
        if (w) {
            write_y(nch - 1);
            float* srow = Sg + (size_t)row * kHd;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float sv[32];
                tmem_ld32(tm + lane_addr + kTmS + c * 32, sv);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4*>(srow + c * 32 + i) =
                        make_float4(sv[i], sv[i + 1], sv[i + 2], sv[i + 3]);
            }
        }
    }
    // do not leave while copies or MMAs this CTA issued may still land
    if (tid == 0) {
        for (int i = 0; i < 8; i++)
            if (out_[i]) mbar_drain(smem_u32(bar_list[i]), par_[i]);
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

// Workspace: fp16 hi+lo planes of q, k (16 heads each) and v (32 heads); f32
// g and beta [B*32][T]; per (sequence, V head, chunk) item the chunk-local
// factors W^T fp16 [128][64], U~^T f32 [64][128], P' fp16 hi/lo [64][64],
// Q~ fp16 [64][128] and K~ fp16 hi/lo [64][128].
struct DnWs {
    size_t qh, ql, kh, kl, vh, vl, g, be, wt, ut, ph, pl, qt, kth, ktl, total;
};

static DnWs dn_ws_layout(int B, int T) {
    auto al = [](size_t x) { return (x + 1023) & ~size_t(1023); };
    const size_t nq = (size_t)B * kNumQK * T * kHd * 2, nv = (size_t)B * kNumV * T * kHd * 2;
    const size_t items = (size_t)B * kNumV * ((T + kC - 1) / kC);
    DnWs w;
    size_t o = 0;
    w.qh = o; o = al(o + nq);
    w.ql = o; o = al(o + nq);
    w.kh = o; o = al(o + nq);
    w.kl = o; o = al(o + nq);
    w.vh = o; o = al(o + nv);
    w.vl = o; o = al(o + nv);
    w.g = o;  o = al(o + (size_t)B * kNumV * T * 4);
    w.be = o; o = al(o + (size_t)B * kNumV * T * 4);
    w.wt = o; o = al(o + items * kHd * kC * 2);
    w.ut = o; o = al(o + items * kHd * kC * 4);
    w.ph = o; o = al(o + items * kC * kC * 2);
    w.pl = o; o = al(o + items * kC * kC * 2);
    w.qt = o; o = al(o + items * kC * kHd * 2);
    w.kth = o; o = al(o + items * kC * kHd * 2);
    w.ktl = o; o = al(o + items * kC * kHd * 2);
    w.total = o;
    return w;
}

size_t dn_prefill_ws_bytes(int batch, int T) { return dn_ws_layout(batch, T).total; }

cudaError_t launch_dn_prefill(qm_ctx* ctx, const qm_dn_params* p, qm_dn_state* st, int T,
                              const uint16_t* qkv, const float* a, const float* bgate, float* y,
                              const float* z, float* out) {
    const int B = st->batch;
    const int nch = (T + kC - 1) / kC;
    cudaStream_t s = ctx->stream;
    const DnWs w = dn_ws_layout(B, T);
    char* base = static_cast<char*>(ctx->ws);
    uint16_t* qh = reinterpret_cast<uint16_t*>(base + w.qh);
    uint16_t* ql = reinterpret_cast<uint16_t*>(base + w.ql);
    uint16_t* kh = reinterpret_cast<uint16_t*>(base + w.kh);
    uint16_t* kl = reinterpret_cast<uint16_t*>(base + w.kl);
    uint16_t* vh = reinterpret_cast<uint16_t*>(base + w.vh);
    uint16_t* vl = reinterpret_cast<uint16_t*>(base + w.vl);
    float* g = reinterpret_cast<float*>(base + w.g);
    float* be = reinterpret_cast<float*>(base + w.be);
    uint16_t* wt = reinterpret_cast<uint16_t*>(base + w.wt);
    float* ut = reinterpret_cast<float*>(base + w.ut);
    uint16_t* ph = reinterpret_cast<uint16_t*>(base + w.ph);
    uint16_t* pl = reinterpret_cast<uint16_t*>(base + w.pl);
    uint16_t* qt = reinterpret_cast<uint16_t*>(base + w.qt);
    uint16_t* kth = reinterpret_cast<uint16_t*>(base + w.kth);
    uint16_t* ktl = reinterpret_cast<uint16_t*>(base + w.ktl);
    {
        TimedLaunch tl(ctx, "dn_prefill_prep");
        const int nruns = (T + kPrepRun - 1) / kPrepRun;
        const size_t warps = (size_t)B * nruns * 64;
        dn_prefill_prep<<<(unsigned)((warps + kPrepWarps - 1) / kPrepWarps), 32 * kPrepWarps, 0, s>>>(
            qkv, a, bgate, p->conv_w, p->a_log, p->dt_bias, st->conv, st->conv_pos, T, nruns, qh, ql, kh,
            kl, vh, vl, g, be, B, ctx->d_err);
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
    const uint64_t items = (uint64_t)B * kNumV * nch;
    CUtensorMap mwt, mph, mpl, mqt, mkth, mktl;
    if (encode_rows_tmap(&mwt, wt, kC, kHd, items, 64, kHd, true) != QM_OK ||
        encode_rows_tmap(&mph, ph, kC, kC, items, 64, kC, true) != QM_OK ||
        encode_rows_tmap(&mpl, pl, kC, kC, items, 64, kC, true) != QM_OK ||
        encode_rows_tmap(&mqt, qt, kHd, kC, items, 64, kC, true) != QM_OK ||
        encode_rows_tmap(&mkth, kth, kHd, kC, items, 64, kC, true) != QM_OK ||
        encode_rows_tmap(&mktl, ktl, kHd, kC, items, 64, kC, true) != QM_OK)
        return cudaErrorInvalidValue;
    static std::atomic<uint64_t> attr_local{0}, attr_state{0};
    e = set_smem_once(attr_local, ctx->device, dn_chunk_local, kLocalSmem);
    if (e == cudaSuccess) e = set_smem_once(attr_state, ctx->device, dn_chunk_state, kStateSmem);
    if (e != cudaSuccess) return e;
    {
        TimedLaunch tl(ctx, "dn_chunk_local");
        dn_chunk_local<<<dim3(kNumV, nch, B), kLocalThreads, kLocalSmem, s>>>(
            m[0], m[1], m[2], m[3], m[4], m[5], g, be, T, nch, wt, ut, ph, pl, qt, kth, ktl, ctx->d_err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    {
        TimedLaunch tl(ctx, "dn_chunk_state");
        dn_chunk_state<<<dim3(kNumV, B), 128, kStateSmem, s>>>(mwt, mph, mpl, mqt, mkth, mktl, ut, g,
                                                               st->s, y, T, nch, ctx->d_err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    if (z) {
        const size_t nh = (size_t)B * T * kNumV;
        dn_prefill_gate<<<(unsigned)((nh + 7) / 8), 256, 0, s>>>(y, z, p->norm_gamma, out, nh);
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
    if ((uintptr_t)qkv & 15) return set_error(c, QM_E_ARG, "qm_dn_prefill: qkv must be 16-byte aligned");
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
