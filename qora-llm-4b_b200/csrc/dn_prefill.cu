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
int encode_f32_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                    uint32_t box_inner, uint32_t box_rows);

namespace {

constexpr int kC = 64;  // chunk length (tokens)
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// prep: one warp per (head-vector, run of kPrepRun tokens, sequence); lane l owns
// the 4 channels 4l..4l+3 of the 128-channel head-vector (8-byte bf16 loads,
// the conv history of those channels kept in registers along the run).
// head-vectors 0..15 = q heads, 16..31 = k heads, 32..63 = v heads
// ---------------------------------------------------------------------------
constexpr int kPrepRun = 12;  // tokens a warp (16: 0.65 ms on workload 2, 12 with 7 CTAs an SM: 0.62)
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

__global__ void __launch_bounds__(32 * kPrepWarps, 7)
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
constexpr uint32_t kIdKK = umma_idesc_f16kind(128, 64, false, false, false);   // A K, B K
constexpr uint32_t kIdW = umma_idesc_f16kind(128, 64, true, false, false);     // A MN, B K

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

// c (a 16 x 8 tile) = X[16 rows][k0, k0 + 8 NK) Y[k0, k0 + 8 NK)[8 columns] for
// f32 X and Y in shared memory (row stride 68 floats), as three TF32 products
// per k-step (hi.hi + hi.lo + lo.hi: about 22 significant bits, f32 range),
// accumulated in three independent chains.  X rows and Y columns start at the
// pointers; k0 is a multiple of 8.  Fragment loads of X touch 32 distinct
// banks (rows 68 floats apart).
template <int NK>
__device__ __forceinline__ void mma3_tf32_tile_n(float (&c)[4], const float* __restrict__ X,
                                                 const float* __restrict__ Y, int k0, int lane) {
    constexpr int S = 68;
    const int g = lane >> 2, t = lane & 3;
    float af[NK][4], bf[NK][2];
#pragma unroll
    for (int s = 0; s < NK; s++) {
        const int k = k0 + 8 * s;
        af[s][0] = X[g * S + k + t];
        af[s][1] = X[(g + 8) * S + k + t];
        af[s][2] = X[g * S + k + t + 4];
        af[s][3] = X[(g + 8) * S + k + t + 4];
        bf[s][0] = Y[(k + t) * S + g];
        bf[s][1] = Y[(k + t + 4) * S + g];
    }
    float ch[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < NK; s++) {
        uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            ah[i] = tf32_rna(af[s][i]);
            al[i] = tf32_rna(af[s][i] - __uint_as_float(ah[i]));
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            bh[i] = tf32_rna(bf[s][i]);
            bl[i] = tf32_rna(bf[s][i] - __uint_as_float(bh[i]));
        }
        mma_tf32_1688(ch, ah[0], ah[1], ah[2], ah[3], bh[0], bh[1]);
        mma_tf32_1688(c1, ah[0], ah[1], ah[2], ah[3], bl[0], bl[1]);
        mma_tf32_1688(c2, al[0], al[1], al[2], al[3], bh[0], bh[1]);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) c[i] = ch[i] + (c1[i] + c2[i]);
}

// the same over nk = 1 .. 4 k-steps (warp-uniform)
__device__ __forceinline__ void mma3_tf32_tile(float (&c)[4], const float* __restrict__ X,
                                               const float* __restrict__ Y, int k0, int k1, int lane) {
    switch ((k1 - k0) >> 3) {
        case 1: mma3_tf32_tile_n<1>(c, X, Y, k0, lane); break;
        case 2: mma3_tf32_tile_n<2>(c, X, Y, k0, lane); break;
        case 3: mma3_tf32_tile_n<3>(c, X, Y, k0, lane); break;
        default: mma3_tf32_tile_n<4>(c, X, Y, k0, lane); break;
    }
}

// stores s * c (a 16 x 8 accumulator tile) at Z (row stride 68 floats)
__device__ __forceinline__ void store_tile_1688(float* __restrict__ Z, const float (&c)[4], float s, int lane) {
    constexpr int S = 68;
    const int g = lane >> 2, t = lane & 3;
    *reinterpret_cast<float2*>(Z + g * S + 2 * t) = make_float2(s * c[0], s * c[1]);
    *reinterpret_cast<float2*>(Z + (g + 8) * S + 2 * t) = make_float2(s * c[2], s * c[3]);
}

struct ChunkBars {
    uint64_t load, mma;
    uint32_t tmem_base;
    int abort_flag;
};

// ---- 2a. chunk-local WY factors: persistent CTAs (8 warps, two per SM) walk
// the (V head, chunk, sequence) items ----
//
// Everything in a chunk that does not depend on the state entering it:
//   MMA1  [K;Q] K^T                       (compensated)  -> A (f32) and P'
//   T = (I + A)^-1 blocked by 16: the diagonal blocks by forward substitution
//         (f32), the blocks below them as 3 x TF32 warp-level MMA tiles
//   MMA2  W^T  = K^T (T diag(b e^G))^T    (compensated)
//   MMA3  U~^T = V^T (T diag(b))^T        (compensated)
// written to the workspace for the state pass: W^T fp16 [128 k][64 t],
// U~^T f32 as [16][128 v][4] (float4 of 4 tokens per v, so the state pass
// loads it with one bulk copy and reads it conflict-free) and P' fp16 hi/lo
// [64 t][64 s]: 64 KB per (chunk, V head).  The state pass uses q and k as
// the prep kernel wrote them (the two V heads of a QK head share them in L2).
// 102 KB of shared memory and 256 TMEM columns a CTA.  Warps w and w+4 share
// TMEM lane quarter w%4 and split the 64 columns of every TMEM tile.
constexpr int kL_KQh = 0;              // [K;Q] hi: 2 boxes [128 rows x 64] fp16 (K rows 0-63,
constexpr int kL_KQl = 32768;          //   Q rows 64-127); once MMA1 is done the four Q
constexpr int kL_Vh = kL_KQh + 8192;   //   quarters take V hi / lo [64 t x 64 v] (the boxes
constexpr int kL_Vl = kL_KQl + 8192;   //   of v columns 64-127 16 KB further on)
constexpr int kAStride = 68;           // floats per A / T row (float4-aligned)
constexpr int kL_A = 65536;            // A f32 [64][68] and T f32 [64][68] during the
constexpr int kL_Tm = kL_A + 64 * kAStride * 4;  // solve, then T' hi/lo over A, T'' hi/lo over T
constexpr int kL_T1h = kL_A, kL_T1l = kL_A + 8192, kL_T2h = kL_Tm, kL_T2l = kL_Tm + 8192;
constexpr int kL_Misc = kL_Tm + 64 * kAStride * 4;  // G, beta, g, b e^G, e^G, e^(G63-G): 6 x 64 f32
constexpr int kLocalSmem = kL_Misc + 6 * 64 * 4 + 64 + 1024;
static_assert(kL_T1l + 8192 <= kL_Tm && kL_T2l + 8192 <= kL_Misc, "T' over A, T'' over T");
static_assert(kL_Tm % 1024 == 0 && kL_T2l % 1024 == 0, "swizzled tiles on 1024-byte boundaries");
constexpr uint32_t kTmKQ = 0, kTmW = 64, kTmU = 128;
constexpr int kLocalThreads = 256;

__global__ void __launch_bounds__(kLocalThreads, 2)
dn_chunk_local(const __grid_constant__ CUtensorMap tqh, const __grid_constant__ CUtensorMap tql,
               const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
               const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
               const __grid_constant__ CUtensorMap tmw,
               const float* __restrict__ gin, const float* __restrict__ bin, int T, int nch, int B,
               uint16_t* __restrict__ wt_out, float* __restrict__ ut_out,
               uint16_t* __restrict__ ph_out, uint16_t* __restrict__ pl_out, int* err) {
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

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;  // TMEM lanes 32*quarter.., columns 32*half..
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int row = quarter * 32 + lane;              // TMEM lane = tile row
    const int nitems = B * kNumV * nch;
    // work item L: V head L % 32 (the two V heads of a QK head side by side, so
    // their K/Q tiles meet in L2), then chunk, then sequence
    auto item_of = [&](int L, int& vh, int& ci, int& b) {
        vh = L % kNumV;
        ci = (L / kNumV) % nch;
        b = L / (kNumV * nch);
    };
    auto load_kq = [&](int vh, int ci, int b) {  // thread 0
        const uint32_t lb = smem_u32(&bars->load);
        const int t0 = ci * kC, plane_qk = b * kNumQK + (vh >> 1);
        mbar_arrive_expect_tx(lb, 8 * 8192);
        for (int hb = 0; hb < 2; hb++) {
            tma_load_3d(sb + kL_KQh + hb * 16384, &tkh, hb * 64, t0, plane_qk, lb);
            tma_load_3d(sb + kL_KQl + hb * 16384, &tkl, hb * 64, t0, plane_qk, lb);
            tma_load_3d(sb + kL_KQh + hb * 16384 + 8192, &tqh, hb * 64, t0, plane_qk, lb);
            tma_load_3d(sb + kL_KQl + hb * 16384 + 8192, &tql, hb * 64, t0, plane_qk, lb);
        }
    };
    auto load_gates = [&](int vh, int ci, int b, float& g, float& be) {
        const int t = ci * kC + tid;
        g = be = 0.f;
        if (tid < kC && t < T) {
            const size_t o = ((size_t)b * kNumV + vh) * T + t;
            g = gin[o];
            be = bin[o];
        }
    };

    // the first item's gates and K/Q tiles arrive while the CTA sets up; each
    // later item's are requested as soon as the previous item's tensor-core
    // work is done, and arrive during its outputs
    int L = blockIdx.x;
    float g_own = 0.f, b_own = 0.f;
    // thread 0's record of the last phase it started on each barrier and not
    // yet seen complete (drained on the way out of an aborted CTA)
    bool ld_out = false, mm_out = false;
    uint32_t ld_par = 0, mm_par = 0;
    {
        int vh, ci, b;
        item_of(L, vh, ci, b);
        if (L < nitems) load_gates(vh, ci, b, g_own, b_own);
        if (tid == 0) {
            mbar_init(smem_u32(&bars->load), 1);
            mbar_init(smem_u32(&bars->mma), 1);
            bars->abort_flag = 0;
            fence_barrier_init();
            if (L < nitems) {
                load_kq(vh, ci, b);
                ld_out = true;
            }
        }
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(&bars->tmem_base), 256);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = bars->tmem_base;
    bool ok = true;

    for (; L < nitems; L += gridDim.x) {
        int vh, ci, b;
        item_of(L, vh, ci, b);
        const int t0 = ci * kC;
        const size_t plane_v = (size_t)b * kNumV + vh;
        const size_t item = ((size_t)b * kNumV + vh) * nch + ci;
        if (tid < kC) {
            sg[tid] = g_own;
            sB[tid] = b_own;
        }
        if (tid == 0) bulk_wait_read0();  // the previous item's W^T store has read the A region
        __syncthreads();
        if (warp == 0) chunk_decays(sg, sG, eG, eD, lane);
        ok = mbar_wait_bounded(smem_u32(&bars->load), 0, abort_flag, err);
        if (ok) ld_out = false;
        ok = __syncthreads_and(ok) != 0;  // also publishes sG
        if (!ok) break;
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
        if (ok && tid == 0) {  // MMA1 has read Q: V lands in its quarters during the solve
            const uint32_t lb = smem_u32(&bars->load);
            mbar_arrive_expect_tx(lb, 4 * 8192);
            ld_out = true;
            ld_par = 1;
            for (int hb = 0; hb < 2; hb++) {
                tma_load_3d(sb + kL_Vh + hb * 16384, &tvh, hb * 64, t0, (int)plane_v, lb);
                tma_load_3d(sb + kL_Vl + hb * 16384, &tvl, hb * 64, t0, (int)plane_v, lb);
            }
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
                if (QM_IN((item * kC + t) * kC + s0, 32, (size_t)nitems * kC * kC, err)) {
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
        tc_fence_before();
        // A is complete once warps 0, 1, 4, 5 (its rows) meet; warps 2, 3, 6, 7
        // go on writing P' while the diagonal blocks are solved
        if (quarter < 2) named_bar_sync(1, 128);

        // ---- T = (I + A)^-1, blocked by 16: diagonal blocks by forward substitution
        // (f32), then the blocks below them from products with T's known blocks ----
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
            } else if (warp == 4 || warp == 5) {
                const int t = tid - 2 * kC;
                sC1[t] = sB[t] * eG[t];
            }
            __syncthreads();
            // the off-diagonal blocks in two levels of 16 x 8 tensor-core tiles
            // (3 x TF32).  Level 1, warps 0-3: for (i, j) = (1, 0), (3, 2),
            // X_ij = A_ij T_jj (kept in the unused block (j, i)), then
            // T_ij = -T_ii X_ij.  Level 2, 8 warps: with T_A, T_B the inverses
            // of the leading and trailing 32 x 32 halves, X = A_BA T_A (kept in
            // rows 0-31, columns 32-63), then T_BA = -T_B X.  k-steps that only
            // meet T's zero upper part (whose storage holds the X's) are skipped.
            static_assert(kAStride == 68, "mma3_tf32_tile assumes the A/T row stride");
            constexpr int S = kAStride;
            if (warp < 4) {
                const int i = 2 * (warp >> 1) + 1, j = i - 1, h = warp & 1;
                float c[4];
                mma3_tf32_tile(c, Amat + 16 * i * S + 16 * j, Tm + 16 * j * S + 16 * j + 8 * h, 8 * h, 16, lane);
                store_tile_1688(Tm + 16 * j * S + 16 * i + 8 * h, c, 1.f, lane);
            }
            __syncthreads();
            if (warp < 4) {
                const int i = 2 * (warp >> 1) + 1, j = i - 1, h = warp & 1;
                float c[4];
                mma3_tf32_tile(c, Tm + 16 * i * S + 16 * i, Tm + 16 * j * S + 16 * i + 8 * h, 0, 16, lane);
                store_tile_1688(Tm + 16 * i * S + 16 * j + 8 * h, c, -1.f, lane);
            }
            __syncthreads();
            {
                const int rt = warp >> 2, ct = warp & 3;
                float c[4];
                mma3_tf32_tile(c, Amat + (32 + 16 * rt) * S, Tm + 8 * ct, 8 * ct, 32, lane);
                store_tile_1688(Tm + 16 * rt * S + 32 + 8 * ct, c, 1.f, lane);
                __syncthreads();
                mma3_tf32_tile(c, Tm + (32 + 16 * rt) * S + 32, Tm + 32 + 8 * ct, 0, rt ? 32 : 16, lane);
                store_tile_1688(Tm + (32 + 16 * rt) * S + 8 * ct, c, -1.f, lane);
            }
            __syncthreads();
            // T' = T diag(b e^G), T'' = T diag(b) as fp16 hi/lo [t][j] tiles (upper
            // part zero), formed in registers and written over A and T once every
            // thread has read its part of T
            static_assert(kC * 8 == 2 * kLocalThreads, "two 8-column pieces of T a thread");
            uint4 t1h[2], t1l[2], t2h[2], t2l[2];
#pragma unroll
            for (int it = 0; it < 2; it++) {
                const int o = tid + it * kLocalThreads, t = o >> 3, j0 = (o & 7) * 8;
                float v1[8], v2[8];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const int j = j0 + q;
                    const float tv = (j <= t) ? Tm[t * kAStride + j] : 0.f;
                    v1[q] = tv * sC1[j];
                    v2[q] = tv * sB[j];
                }
                split8(v1, t1h[it], t1l[it]);
                split8(v2, t2h[it], t2l[it]);
            }
            __syncthreads();
#pragma unroll
            for (int it = 0; it < 2; it++) {
                const int o = tid + it * kLocalThreads;
                const uint32_t so = sw128_off(o >> 3, o & 7);
                *reinterpret_cast<uint4*>(smem + kL_T1h + so) = t1h[it];
                *reinterpret_cast<uint4*>(smem + kL_T1l + so) = t1l[it];
                *reinterpret_cast<uint4*>(smem + kL_T2h + so) = t2h[it];
                *reinterpret_cast<uint4*>(smem + kL_T2l + so) = t2l[it];
            }
        }
        fence_proxy_async_shared();  // the T tiles, for the tensor core
        tc_fence_before();
        __syncthreads();

        // ---- MMA2 (W^T) now, MMA3 (U~^T) once V has landed ----
        if (ok && tid == 0) {
            const uint32_t lb = smem_u32(&bars->load);
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
                        umma_bf16_ss(tm + kTmU, umma_sdesc(va + kk * 2048, 16384, 1024),
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
        if (!ok) break;

        // the next item's K/Q tiles (the region is free: MMA2/3 are done) and gates
        if (L + (int)gridDim.x < nitems) {
            int vh2, ci2, b2;
            item_of(L + gridDim.x, vh2, ci2, b2);
            load_gates(vh2, ci2, b2, g_own, b_own);
            if (tid == 0) {
                load_kq(vh2, ci2, b2);
                ld_out = true;
                ld_par = 0;
            }
        }

        // ---- outputs: W^T row k (fp16) through the A region (free since MMA2/3)
        // and one TMA store; U~^T row v (f32, [t/4][v][4]) straight to global.
        // This thread's 32 tokens [32 half, 32 half + 32) ----
        {
            float wv[32];
            tmem_ld32(tm + lane_addr + kTmW + half * 32, wv);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; t += 8)
                *reinterpret_cast<uint4*>(smem + kL_A + sw128_off(row, half * 4 + t / 8)) = round8(wv + t);
        }
        fence_proxy_async_shared();
        __syncthreads();
        if (tid == 0 && QM_IN(item * kHd * kC, kHd * kC, (size_t)nitems * kHd * kC, err)) {
            tma_store_3d(&tmw, sb + kL_A, 0, 0, (int)item);
            bulk_commit();
        }
        if (QM_IN(item * kHd * kC, kHd * kC, (size_t)nitems * kHd * kC, err)) {
            float uv[32];
            tmem_ld32(tm + lane_addr + kTmU + half * 32, uv);
            tmem_ld_wait();
            float4* ub = reinterpret_cast<float4*>(ut_out + item * kHd * kC);
#pragma unroll
            for (int i = 0; i < 8; i++)
                ub[(half * 8 + i) * kHd + row] = make_float4(uv[4 * i], uv[4 * i + 1], uv[4 * i + 2], uv[4 * i + 3]);
        }
        tc_fence_before();
    }  // items

    if (tid == 0) {
        bulk_wait0();  // every W^T store has completed
        if (ld_out) mbar_drain(smem_u32(&bars->load), ld_par, err);
        if (mm_out) mbar_drain(smem_u32(&bars->mma), mm_par, err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tm, 256);
    }
}

// ---- 2b. state pass: one CTA per (V head, sequence), 12 warps ----
//
// Per chunk c, with S0 the state entering it (f32 master in TMEM, and an fp16
// copy in TMEM as the A operand), G the in-chunk cumulative log-decay,
// D_s = e^(G63 - G_s) and q, k the prep kernel's fp16 hi/lo tiles:
//   MMA4  U = U~ - S0 W^T  (U~ preloaded into U2[c&1])
//   MMA7  S += (U diag D)^T k  (compensated; S pre-scaled by e^G63)
//   MMA5  Y1 = S0 q_hi^T       MMA6  Y2 = U^T P'^T (compensated)
//   y_t = e^G_t Y1_t + Y2_t;   S0 (fp16, TMEM buffer (c+1)&1) = S
// The decays fold into the operands the chain already touches (the U step
// scales U's columns before splitting it into fp16 hi/lo, the readout
// scales Y1), so q and k are used as the prep kernel wrote them.
// Warps 0-3 (lane = v row) run the chain MMA4 -> U step -> MMA7 -> S pass
// (the fp16 S0 of the next chunk, and S scaled by that chunk's e^G63 for its
// MMA7, in one read of S); thread 0 issues MMA4, MMA7 and the W^T and k
// loads.  Warps 4-7 run beside it: each chunk's decays, U~ of the next chunk
// into TMEM, the unscaled U hi/lo for MMA6; their thread 128 issues MMA5 /
// MMA6.  Warps 8-11 wait for those, write y (staged in shared memory, TMA
// stores of half chunks) and their thread 256 issues the next q and P'
// loads.  mbarriers hand over: u2_ready, dec_ready (warps 4-7 -> thread 0);
// u_ready, s_read (thread 0 -> warps 4-7); y_free (warps 8-11 -> warps 4-7,
// which also frees U^T hi/lo and q for reuse).  u2_ready, dec_ready, s_read
// and mY are pairs used by chunk parity (phase c >> 1 for chunk c): either
// side may publish a chunk's piece one chunk early without a phase running
// two ahead of its waiter.
constexpr int kS_W = 0;             // W^T [128 k x 64 t] fp16 (16 KB)
constexpr int kS_Q = 16384;         // q hi [64 t x 128 k] fp16: 2 boxes [64 x 64], x2 buffers (32 KB)
constexpr int kS_P = 49152;         // P' hi, lo [64 t x 64 s] (8 KB each) (16 KB)
constexpr int kS_K = 65536;         // k hi, lo [64 s x 128 k] (16 KB each), x2 buffers (64 KB)
constexpr int kS_Us = 131072;       // (U diag D)^T hi, lo [128 v x 64 s] (16 KB each)
constexpr int kS_Uu = 163840;       // U^T hi, lo (16 KB each)
constexpr int kS_Y = 196608;        // y staging, half a chunk: [32 t][128 v] f32 (16 KB)
constexpr int kS_Misc = 212992;     // [4] x (g, G, eG, eD): 16 x 64 f32; barriers
constexpr int kMiscSlots = 4;       // chunk c's decays in slot c & 3
constexpr int kStateSmem = kS_Misc + kMiscSlots * 4 * 64 * 4 + 256 + 1024;
// TMEM columns: S f32 [0,128), S0 fp16 pairs x2 [128,256), U2 f32 x2 [256,384), Y1 [384,448), Y2 [448,512)
constexpr uint32_t kTmS = 0, kTmS0h = 128, kTmU2 = 256, kTmY1 = 384, kTmY2 = 448;
constexpr uint32_t kNegB = 1u << 14;
constexpr uint32_t kIdSW = umma_idesc_f16kind(128, 64, false, true, false) | kNegB;  // A tmem, -B(MN)
constexpr uint32_t kIdSQ = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUP = umma_idesc_f16kind(128, 64, false, false, false);
constexpr uint32_t kIdUK = umma_idesc_f16kind(128, 128, false, true, false);   // A K, B MN

struct StateBars {  // the first 11 words are tracked by Pending (in this order)
    uint64_t w_full[2], q_full[2], k_full[2], p_full;  // TMA
    uint64_t m4, m7, mY[2];                            // MMA completions (mY: a chunk-parity pair)
    uint64_t u2_ready[2], dec_ready[2];                // warps 4-7 -> thread 0 (128 arrivals)
    uint64_t u_ready, s_read[2];                       // thread 0 -> warps 4-7 (1 arrival)
    uint64_t y_free;                                   // warps 8-11 read Y out (128 arrivals)
    uint32_t tmem_base;
    int abort_flag;
};

// bar.red.and over named barrier `id` of `count` threads
__device__ __forceinline__ bool named_bar_and(int id, int count, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

// The issuing thread's record of barrier phases it started and has not yet
// seen complete (one bit per barrier among the first 11 words of StateBars),
// drained on the way out so nothing lands after the CTA ends.
struct Pending {
    uint64_t* base;
    uint32_t out = 0, par = 0;
    __device__ explicit Pending(uint64_t* b) : base(b) {}
    __device__ void start(uint64_t* b, uint32_t parity) {
        const uint32_t bit = 1u << (uint32_t)(b - base);
        out |= bit;
        par = parity ? (par | bit) : (par & ~bit);
    }
    __device__ void seen(uint64_t* b) { out &= ~(1u << (uint32_t)(b - base)); }
    __device__ void drain(int* err) {
        for (int i = 0; i < 11; i++)
            if (out & (1u << i)) mbar_drain(smem_u32(base + i), (par >> i) & 1u, err);
    }
};

// U (64 f32 of one v row, token order) -> fp16 hi/lo, K-major swizzled rows
__device__ __forceinline__ void store_u_split(uint8_t* smem_hi, uint8_t* smem_lo, int row, const float* u) {
#pragma unroll
    for (int s = 0; s < kC; s += 8) {
        uint4 h, l;
        split8(u + s, h, l);
        *reinterpret_cast<uint4*>(smem_hi + sw128_off(row, s >> 3)) = h;
        *reinterpret_cast<uint4*>(smem_lo + sw128_off(row, s >> 3)) = l;
    }
}

constexpr int kStateThreads = 384;  // warps 0-3: the recurrence; 4-7: beside it; 8-11: y

__global__ void __launch_bounds__(kStateThreads, 1)
dn_chunk_state(const __grid_constant__ CUtensorMap twt, const __grid_constant__ CUtensorMap tph,
               const __grid_constant__ CUtensorMap tpl, const __grid_constant__ CUtensorMap tqh,
               const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
               const __grid_constant__ CUtensorMap tyo,
               const float* __restrict__ ut_in, const float* __restrict__ gin,
               float* __restrict__ S, int T, int nch, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* misc = reinterpret_cast<float*>(smem + kS_Misc);  // slot s: g, G, eG, eD at misc + 256 s
    StateBars* bars = reinterpret_cast<StateBars*>(misc + kMiscSlots * 256);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sb = smem_u32(smem);

    const int vh = blockIdx.x, b = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = tid & 127;  // TMEM lane = v row
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const size_t plane_v = (size_t)b * kNumV + vh;
    const int plane_qk = b * kNumQK + (vh >> 1);  // the prep kernel's q/k planes
    const size_t item0 = plane_v * nch;

    if (tid == 0) {
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&bars->w_full[i]), 1);
            mbar_init(smem_u32(&bars->q_full[i]), 1);
            mbar_init(smem_u32(&bars->k_full[i]), 1);
        }
        mbar_init(smem_u32(&bars->p_full), 1);
        mbar_init(smem_u32(&bars->m4), 1);
        mbar_init(smem_u32(&bars->m7), 1);
        mbar_init(smem_u32(&bars->mY[0]), 1);
        mbar_init(smem_u32(&bars->mY[1]), 1);
        mbar_init(smem_u32(&bars->u2_ready[0]), 128);
        mbar_init(smem_u32(&bars->u2_ready[1]), 128);
        mbar_init(smem_u32(&bars->dec_ready[0]), 128);
        mbar_init(smem_u32(&bars->dec_ready[1]), 128);
        mbar_init(smem_u32(&bars->u_ready), 1);
        mbar_init(smem_u32(&bars->s_read[0]), 1);
        mbar_init(smem_u32(&bars->s_read[1]), 1);
        mbar_init(smem_u32(&bars->y_free), 128);
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
    Pending pend(&bars->w_full[0]);
    auto wait = [&](uint64_t* bar, uint32_t parity) {
        const bool w = mbar_wait_bounded(smem_u32(bar), parity, abort_flag, err);
        if (w) pend.seen(bar);
        return w;
    };

    // ---- loads (thread 0: W^T, k; thread 128: q, P') ----
    auto issue_w = [&](int c) {  // W^T of chunk c (one buffer: loaded as soon as MMA4 of c-1 is done)
        uint64_t* fb = &bars->w_full[0];
        pend.start(fb, c & 1);
        mbar_arrive_expect_tx(smem_u32(fb), 16384);
        tma_load_3d(sb + kS_W, &twt, 0, 0, (int)(item0 + c), smem_u32(fb));
    };
    auto issue_q = [&](int c) {  // q hi of chunk c into buffer c & 1
        uint64_t* fb = &bars->q_full[c & 1];
        pend.start(fb, (c >> 1) & 1);
        mbar_arrive_expect_tx(smem_u32(fb), 16384);
        for (int hb = 0; hb < 2; hb++)
            tma_load_3d(sb + kS_Q + (c & 1) * 16384 + hb * 8192, &tqh, hb * 64, c * kC, plane_qk, smem_u32(fb));
    };
    auto issue_k = [&](int c) {  // k hi/lo of chunk c into buffer c & 1
        uint64_t* fb = &bars->k_full[c & 1];
        pend.start(fb, (c >> 1) & 1);
        mbar_arrive_expect_tx(smem_u32(fb), 2 * 16384);
        const uint32_t kb = sb + kS_K + (c & 1) * 32768;
        for (int hb = 0; hb < 2; hb++) {
            tma_load_3d(kb + hb * 8192, &tkh, hb * 64, c * kC, plane_qk, smem_u32(fb));
            tma_load_3d(kb + 16384 + hb * 8192, &tkl, hb * 64, c * kC, plane_qk, smem_u32(fb));
        }
    };
    auto issue_p = [&](int c) {  // P' hi/lo of chunk c
        uint64_t* fb = &bars->p_full;
        pend.start(fb, c & 1);
        mbar_arrive_expect_tx(smem_u32(fb), 2 * 8192);
        tma_load_3d(sb + kS_P, &tph, 0, 0, (int)(item0 + c), smem_u32(fb));
        tma_load_3d(sb + kS_P + 8192, &tpl, 0, 0, (int)(item0 + c), smem_u32(fb));
    };
    if (tid == 0) {
        issue_w(0);
        issue_k(0);
        if (nch > 1) issue_k(1);
    }
    if (tid == 128) {
        issue_q(0);
        if (nch > 1) issue_q(1);
        issue_p(0);
    }
    float* Sg = S + (QM_IN(plane_v * kHd * kHd, kHd * kHd, (size_t)gridDim.x * gridDim.y * kHd * kHd, err)
                         ? plane_v * kHd * kHd : 0);

    if (warp < 4) {
        // ================= warps 0-3: the recurrence =================
        bool ok = mbar_wait_bounded(smem_u32(&bars->dec_ready[0]), 0, abort_flag, err);
        {   // initial state: global f32 -> its fp16 copy (S0 buffer 0) and, scaled by
            // e^G63 of chunk 0 for MMA7, the TMEM master
            const float* srow = Sg + (size_t)row * kHd;
            const float decay = misc[128 + kC - 1];
#pragma unroll 1
            for (int h = 0; h < 2; h++) {
                float pk[32];
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const int c = 2 * h + cc;
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        const float4 f = *reinterpret_cast<const float4*>(srow + c * 32 + i);
                        v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
                    }
#pragma unroll
                    for (int i = 0; i < 16; i++) pk[cc * 16 + i] = __uint_as_float(pack_f16x2_rn(v[2 * i], v[2 * i + 1]));
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] *= decay;
                    tmem_st32(tm + lane_addr + kTmS + c * 32, v);
                }
                tmem_st32(tm + lane_addr + kTmS0h + h * 32, pk);
            }
            tmem_st_wait();
        }
        tc_fence_before();
        ok = named_bar_and(1, 128, ok);
        if (tid == 0) mbar_arrive(smem_u32(&bars->s_read[0]));  // S0 of chunk 0

        for (int ci = 0; ci < nch && ok; ci++) {
            const int p = ci & 1;
            // ---- MMA4: U2[p] (= U~) -= S0[p] W^T ----
            if (tid == 0) {
                const bool w = wait(&bars->w_full[0], p) && wait(&bars->u2_ready[p], (ci >> 1) & 1);
                tc_fence_after();
                if (w) {
                    for (int kk = 0; kk < 8; kk++)
                        umma_f16_ts(tm + kTmU2 + p * 64, tm + kTmS0h + p * 64 + kk * 8,
                                    umma_sdesc(sb + kS_W + kk * 2048, 8192, 1024), kIdSW, 1u);
                }
                umma_commit(smem_u32(&bars->m4));
                pend.start(&bars->m4, p);
            }
            {
                const bool w = mbar_wait_bounded(smem_u32(&bars->m4), p, abort_flag, err);
                if (tid == 0 && w) pend.seen(&bars->m4);
                ok = named_bar_and(1, 128, ok && w && !*abort_flag);
            }
            if (!ok) break;
            tc_fence_after();
            if (tid == 0 && ci + 1 < nch) issue_w(ci + 1);  // MMA4 has read W^T

            // ---- U step: (U diag D)^T -> fp16 hi/lo (MMA7 of chunk ci-1 is done with them) ----
            {
                float u[64];
                tmem_ld32(tm + lane_addr + kTmU2 + p * 64, u);
                tmem_ld32(tm + lane_addr + kTmU2 + p * 64 + 32, u + 32);
                const float* eD = misc + (ci & 3) * 256 + 192;
                tmem_ld_wait();
#pragma unroll
                for (int s = 0; s < kC; s += 2) {  // packed f32x2 multiplies, two columns an instruction
                    const float2 v = __fmul2_rn(make_float2(u[s], u[s + 1]), *reinterpret_cast<const float2*>(eD + s));
                    u[s] = v.x;
                    u[s + 1] = v.y;
                }
                store_u_split(smem + kS_Us, smem + kS_Us + 16384, row, u);
            }
            fence_proxy_async_shared();
            tc_fence_before();
            named_bar_sync(1, 128);

            // ---- MMA7: S (pre-scaled by e^G63) += (U diag D)^T k ----
            if (tid == 0) {
                mbar_arrive(smem_u32(&bars->u_ready));  // U is read; the chunk's decays are consumed
                const bool w = wait(&bars->k_full[p], (ci >> 1) & 1);
                tc_fence_after();
                if (w) {
                    const uint32_t kb = sb + kS_K + p * 32768;
                    for (int term = 0; term < 3; term++) {
                        const uint32_t ua = sb + kS_Us + (term == 2 ? 16384 : 0);
                        const uint32_t kt = kb + (term == 1 ? 16384 : 0);
                        for (int kk = 0; kk < 4; kk++)
                            umma_bf16_ss(tm + kTmS, umma_sdesc(ua + kk * 32, 16, 1024),
                                         umma_sdesc(kt + kk * 2048, 8192, 1024), kIdUK, 1u);
                    }
                }
                umma_commit(smem_u32(&bars->m7));
                pend.start(&bars->m7, p);
            }
            {
                const bool w = mbar_wait_bounded(smem_u32(&bars->m7), p, abort_flag, err);
                if (tid == 0 && w) pend.seen(&bars->m7);
                ok = named_bar_and(1, 128, ok && w && !*abort_flag);
            }
            if (!ok) break;
            tc_fence_after();
            if (tid == 0 && ci + 2 < nch) issue_k(ci + 2);  // MMA7 has read k buffer p

            // ---- S pass: S0 of chunk ci+1 = fp16(S) into TMEM buffer p^1, and S scaled
            // by e^G63 of chunk ci+1 for its MMA7 (its decays come with dec_ready) ----
            if (ci + 1 < nch) {
                // dec_ready[c&1] completes once per two chunks: phase (c >> 1) for chunk c;
                // MMA5 of chunk ci-1 (mY) has read S0 buffer p^1
                ok = mbar_wait_bounded(smem_u32(&bars->dec_ready[(ci + 1) & 1]), ((ci + 1) >> 1) & 1, abort_flag, err);
                if (ok && ci > 0)
                    ok = mbar_wait_bounded(smem_u32(&bars->mY[(ci - 1) & 1]), ((ci - 1) >> 1) & 1, abort_flag, err);
                const float decay = misc[((ci + 1) & 3) * 256 + 128 + kC - 1];
#pragma unroll 1
                for (int h = 0; h < 2; h++) {
                    float sv[64], pk[32];
                    tmem_ld32(tm + lane_addr + kTmS + h * 64, sv);
                    tmem_ld32(tm + lane_addr + kTmS + h * 64 + 32, sv + 32);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; i++) pk[i] = __uint_as_float(pack_f16x2_rn(sv[2 * i], sv[2 * i + 1]));
                    tmem_st32(tm + lane_addr + kTmS0h + (p ^ 1) * 64 + h * 32, pk);
#pragma unroll
                    for (int i = 0; i < 64; i += 2) {
                        const float2 v = __fmul2_rn(make_float2(sv[i], sv[i + 1]), make_float2(decay, decay));
                        sv[i] = v.x;
                        sv[i + 1] = v.y;
                    }
                    tmem_st32(tm + lane_addr + kTmS + h * 64, sv);
                    tmem_st32(tm + lane_addr + kTmS + h * 64 + 32, sv + 32);
                }
                tmem_st_wait();
            }
            tc_fence_before();
            named_bar_sync(1, 128);
            // S0 of ci+1 written: s_read[(ci+1)&1], whose previous phase (chunk ci-1)
            // warps 4-7 consumed before they published U~ of chunk ci
            if (tid == 0 && ci + 1 < nch) mbar_arrive(smem_u32(&bars->s_read[(ci + 1) & 1]));
            ok = named_bar_and(1, 128, ok && !*abort_flag);
        }
        // ---- final state back to global (f32); warps 4-7 write the last y ----
        if (ok) {
            tc_fence_after();
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
    } else if (warp < 8) {
        // ================= warps 4-7: beside the chain =================
        // Every thread here runs every step (the named barriers need all 128);
        // after an abort the bounded waits return at once and the work is skipped.
        const int at = tid - 128;
        bool ok = true;
        const float* ut_base = ut_in + item0 * kHd * kC;
        const bool ut_in_range =
            QM_IN(item0 * kHd * kC, (size_t)nch * kHd * kC, (size_t)gridDim.x * gridDim.y * nch * kHd * kC, err);
        float ut[64];  // U~ of the next chunk for this thread's v row
        auto load_ut = [&](int c) {
            const float4* ub = reinterpret_cast<const float4*>(ut_base + (size_t)c * kHd * kC);
#pragma unroll
            for (int t4 = 0; t4 < kC / 4; t4++) {
                const float4 f = ut_in_range ? ub[t4 * kHd + row] : make_float4(0.f, 0.f, 0.f, 0.f);
                ut[4 * t4] = f.x; ut[4 * t4 + 1] = f.y; ut[4 * t4 + 2] = f.z; ut[4 * t4 + 3] = f.w;
            }
        };
        auto store_ut = [&](int c) {  // U~ of chunk c into U2[c&1], then u2_ready[c&1]
            tmem_st32(tm + lane_addr + kTmU2 + (c & 1) * 64, ut);
            tmem_st32(tm + lane_addr + kTmU2 + (c & 1) * 64 + 32, ut + 32);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->u2_ready[c & 1]));
        };
        float g_next = 0.f;
        auto load_g = [&](int c) {
            const int t = c * kC + at;
            g_next = (at < kC && c < nch && t < T) ? gin[plane_v * T + t] : 0.f;
        };
        auto decays = [&](int c) {  // the gates of chunk c (in g_next) -> slot c&1, then dec_ready[c&1]
            float* sgp = misc + (c & 3) * 256;
            if (at < kC) sgp[at] = g_next;
            named_bar_sync(2, 128);
            if (warp == 4) chunk_decays(sgp, sgp + 64, sgp + 128, sgp + 192, lane);
            named_bar_sync(2, 128);
            mbar_arrive(smem_u32(&bars->dec_ready[c & 1]));
        };
        // ---- before chunk 0: its decays, U~ -> U2[0] ----
        load_g(0);
        load_ut(0);
        decays(0);
        load_g(1);
        store_ut(0);
        if (nch > 1) load_ut(1);

        for (int ci = 0; ci < nch; ci++) {
            const int p = ci & 1;
            const bool more = ci + 1 < nch;
            // ---- the decays of chunk ci+1 first: the S pass of chunk ci waits for them.
            // Slot (ci+1)&3 was last read for chunk ci-3 (its y read out before MMA5 of
            // ci-1 began); dec_ready[(ci+1)&1] last completed for chunk ci-1, whose S
            // pass waited for it before the U step of ci ----
            if (more) {
                decays(ci + 1);
                load_g(ci + 2);
            }
            // ---- MMA5: Y1 = S0 q^T, once warps 8-11 have read Y of chunk ci-1 ----
            bool qok = ok && wait(&bars->q_full[p], (ci >> 1) & 1);
            if (at == 0) {
                if (ci > 0) qok = qok && mbar_wait_bounded(smem_u32(&bars->y_free), (ci - 1) & 1, abort_flag, err);
                qok = qok && mbar_wait_bounded(smem_u32(&bars->s_read[p]), (ci >> 1) & 1, abort_flag, err);  // S0 of ci
            }
            tc_fence_before();
            named_bar_sync(2, 128);
            if (at == 0) {
                tc_fence_after();
                if (qok) {
                    for (int kk = 0; kk < 8; kk++)
                        umma_f16_ts(tm + kTmY1, tm + kTmS0h + p * 64 + kk * 8,
                                    umma_sdesc(sb + kS_Q + p * 16384 + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                                    kIdSQ, kk > 0 ? 1u : 0u);
                }
            }
            // ---- once the U step of ci is done: U^T hi/lo (unscaled) for MMA6 ----
            const bool wu = mbar_wait_bounded(smem_u32(&bars->u_ready), p, abort_flag, err);
            ok = ok && wu;
            if (ok) {
                tc_fence_after();
                float u[64];
                tmem_ld32(tm + lane_addr + kTmU2 + p * 64, u);
                tmem_ld32(tm + lane_addr + kTmU2 + p * 64 + 32, u + 32);
                tmem_ld_wait();
                store_u_split(smem + kS_Uu, smem + kS_Uu + 16384, row, u);
                fence_proxy_async_shared();
            }
            tc_fence_before();
            named_bar_sync(2, 128);
            if (at == 0) {
                const bool pok = ok && wait(&bars->p_full, p);
                tc_fence_after();
                if (pok) {
                    int n = 0;
                    for (int term = 0; term < 3; term++) {
                        const uint32_t ua = sb + kS_Uu + (term == 2 ? 16384 : 0);
                        const uint32_t pbt = sb + kS_P + (term == 1 ? 8192 : 0);
                        for (int kk = 0; kk < 4; kk++, n++)
                            umma_bf16_ss(tm + kTmY2, umma_sdesc(ua + kk * 32, 16, 1024),
                                         umma_sdesc(pbt + kk * 32, 16, 1024), kIdUP, n > 0 ? 1u : 0u);
                    }
                }
                umma_commit(smem_u32(&bars->mY[p]));  // MMA5 and MMA6 of ci
                pend.start(&bars->mY[p], (ci >> 1) & 1);
            }
            if (more) {
                store_ut(ci + 1);  // U2[(ci+1)&1] was read in chunk ci-1
                if (ci + 2 < nch) load_ut(ci + 2);
            }
            // (the next q and P' loads are issued by warps 8-11 once MMA5/MMA6 are
            // done; U^T hi/lo is rewritten only after y_free of ci, which follows them)
            ok = ok && !*abort_flag;
        }
    } else {
        // ================= warps 8-11: y =================
        // Per chunk: wait for MMA5/MMA6, read Y1 and Y2 from TMEM, form
        // y_t = e^G_t Y1_t + Y2_t (the decays are read before y_free releases Y,
        // which bounds how far warps 4-7 can reuse their slot), then write it in
        // two halves of 32 tokens through a 16 KB staging buffer and TMA stores
        // (tokens past T lie outside the tensor map and are not written).
        const int yt = tid - 256;
        bool ok = true;
        for (int ci = 0; ci < nch; ci++) {
            const bool wy = ok && wait(&bars->mY[ci & 1], (ci >> 1) & 1);
            ok = wy && !*abort_flag;
            if (yt == 0 && ok) {  // MMA6 of ci has read P', MMA5 of ci q buffer ci&1
                if (ci + 1 < nch) issue_p(ci + 1);
                if (ci + 2 < nch) issue_q(ci + 2);
            }
            float yv[64];
            if (wy) {
                tc_fence_after();
                float y2[64];
                tmem_ld32(tm + lane_addr + kTmY1, yv);
                tmem_ld32(tm + lane_addr + kTmY1 + 32, yv + 32);
                tmem_ld32(tm + lane_addr + kTmY2, y2);
                tmem_ld32(tm + lane_addr + kTmY2 + 32, y2 + 32);
                tmem_ld_wait();
                const float* eG = misc + (ci & 3) * 256 + 128;
#pragma unroll
                for (int t = 0; t < kC; t++) yv[t] = fmaf(eG[t], yv[t], y2[t]);
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->y_free));
            float* ys = reinterpret_cast<float*>(smem + kS_Y);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (yt == 0) bulk_wait_read0();  // the previous store has read the buffer
                named_bar_sync(3, 128);
                if (wy) {
#pragma unroll
                    for (int t = 0; t < kC / 2; t++) ys[t * kHd + row] = yv[32 * h + t];
                }
                fence_proxy_async_shared();
                named_bar_sync(3, 128);
                if (yt == 0 && wy) {
                    tma_store_3d(&tyo, sb + kS_Y, vh * kHd, ci * kC + 32 * h, b);
                    bulk_commit();
                }
            }
        }
        if (yt == 0) bulk_wait0();  // the last y stores have completed
    }
    // do not leave while copies or MMAs this CTA issued may still land
    pend.drain(err);
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
// factors W^T fp16 [128][64], U~^T f32 [64][128] and P' fp16 hi/lo [64][64].
struct DnWs {
    size_t qh, ql, kh, kl, vh, vl, g, be, wt, ut, ph, pl, total;
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
    CUtensorMap mwt, mph, mpl, myo;
    if (encode_rows_tmap(&mwt, wt, kC, kHd, items, 64, kHd, true) != QM_OK ||
        encode_rows_tmap(&mph, ph, kC, kC, items, 64, kC, true) != QM_OK ||
        encode_rows_tmap(&mpl, pl, kC, kC, items, 64, kC, true) != QM_OK ||
        encode_f32_tmap(&myo, y, kVDim, (uint64_t)T, (uint64_t)B, kHd, kC / 2) != QM_OK)
        return cudaErrorInvalidValue;
    static std::atomic<uint64_t> attr_local{0}, attr_state{0};
    e = set_smem_once(attr_local, ctx->device, dn_chunk_local, kLocalSmem);
    if (e == cudaSuccess) e = set_smem_once(attr_state, ctx->device, dn_chunk_state, kStateSmem);
    if (e != cudaSuccess) return e;
    {
        TimedLaunch tl(ctx, "dn_chunk_local");
        const int nitems = B * kNumV * nch;  // persistent: two CTAs per SM walk the items
        const int grid = std::min(nitems, 2 * std::max(ctx->num_sms, 1));
        dn_chunk_local<<<grid, kLocalThreads, kLocalSmem, s>>>(m[0], m[1], m[2], m[3], m[4], m[5], mwt, g, be,
                                                               T, nch, B, wt, ut, ph, pl, ctx->d_err);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ctx->launches += 1;
    {
        TimedLaunch tl(ctx, "dn_chunk_state");
        dn_chunk_state<<<dim3(kNumV, B), kStateThreads, kStateSmem, s>>>(mwt, mph, mpl, m[0], m[2], m[3], myo, ut, g,
                                                               st->s, T, nch, ctx->d_err);
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
