// Prefill projections: Y[T][n] = X[T][k] . W for Q4 or F16 weights over a
// whole prompt (the reference's gemm -> gemm_q4 / gemm_f16, src/gemv.rs:294-300,
// 390, 529, used by its prefill at src/gemv.rs:1114-1117, 1222 and 1366-1385).
// At T tokens each weight is reused T times, so this is a tensor-core GEMM,
// not a stream.
//
// qm_gemm_kernel: one CTA per 256 x 256 tile of Y, K in steps of 64.
//  * warp 0 (one thread) loads X tiles [2 x 128 tokens x 64 k] bf16 with TMA
//    (128-byte swizzle: the K-major A operand);
//  * warps 2-11 dequantise the matching W tile [64 k x 256 n] from the
//    reference's Q4 layout (packed nibbles [k][n/2], f16 scales [k][n/32])
//    to bf16 s (q - 8) (the next two stages' words in flight while one is
//    converted; two nibbles a LOP3 as bf16x2 128 + q, minus 136, times the
//    scale in bf16, the columns of each 8 stored in the order 0 4 1 5 2 6 3 7
//    and put back by the epilogue; F16 weights: 8 f16 a 16-byte load, each
//    rounded to the nearest bf16, in column order), written into shared
//    memory in the layout a
//    128-byte-swizzled TMA box of [64 k rows x 64 n] would have (the
//    MN-major B operand: 4 boxes for 256 columns);
//  * warp 1 allocates all 512 TMEM columns (two accumulators of 128 lanes x
//    256 f32, one per half of the 256 rows) and one thread issues
//    tcgen05.mma (kind::f16, bf16 x bf16 -> f32, M 128, N 256, K 16) twice
//    per k-step, both halves reading the same dequantised B, so each W tile
//    is dequantised once for 256 rows; each stage is released to the
//    producers by tcgen05.commit;
//  * warps 4-7 read D out of TMEM (their lane quarters) and store Y (f32 or bf16).
// When the tiles would fill less than half the SMs (a short prompt, a narrow
// weight), K is split over up to 4 CTAs a tile: each stores its f32 partial
// tile to a scratch area and the last to finish (an acquire-release counter)
// adds the partials in split order and stores Y, so the result does not
// depend on timing.  A tile whose second 128 rows all lie past T loads and
// multiplies only its first half.
// A ring of 3 stages (64 KB each) keeps loads, dequantisation and MMAs
// overlapped.  Every wait is bounded: on a timeout the kernel sets the
// context's error word and an abort flag, the TMA thread waits (bounded) for
// its copies in flight, and TMEM is freed before the CTA leaves.
// W in bf16 (the scale rounded to bf16, then the product) carries 8 bits of
// mantissa: max|y - y_exact| / RMS(y) stays within a few 1e-3 (the prefill
// tolerance is 2e-2).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <atomic>
#include <type_traits>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {
int encode_rows_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                     uint32_t box_inner, uint32_t box_rows, bool fp16);
namespace {

constexpr int kGmBM = 256, kGmBN = 256, kGmBK = 64, kGmStages = 3;
constexpr int kGmXBox = 128 * 128;               // [128 rows x 64 bf16] = 16 KB (two a stage)
constexpr int kGmWBox = kGmBK * 128;             // [64 k rows x 64 n bf16] = 8 KB
constexpr int kGmStage = 2 * kGmXBox + 4 * kGmWBox;  // 64 KB
constexpr int kGmOffBar = kGmStages * kGmStage;  // 192 KB
constexpr int kGmSmem = kGmOffBar + 256 + 1024;  // + barriers + alignment slack
constexpr int kGmThreads = 384;
constexpr int kGmProdWarps = 10;  // warps 2..11
constexpr int kGmChunks = (kGmBK * (kGmBN / 8) + kGmProdWarps * 32 - 1) / (kGmProdWarps * 32);  // 7 a thread
constexpr int kGmTmCols = 512;    // two accumulators of 128 lanes x 256 f32
constexpr int kGmMaxSplits = 4;  // split-K: CTAs a tile at most
constexpr uint32_t kGmIdesc = umma_idesc_bf16(128, kGmBN, false, true);      // A K-major, B MN-major
constexpr uint32_t kGmIdescRows = umma_idesc_bf16(128, kGmBN, false, false); // A and B K-major

struct GmBars {
    uint64_t x_full[kGmStages], w_full[kGmStages], free_[kGmStages], done;
    uint32_t tmem_base;
    int abort_flag;
    int last;  // split-K: this CTA is the tile's last to finish and adds the partials
};
static_assert(sizeof(GmBars) <= 256, "barrier block");

// ROWS: W stored one row per output (QM_W_Q4_ROWS, the tied embedding as
// lm_head: packed [n][k/2], scales [n][k/32]) -> B is K-major, one 256-row
// swizzled box, k kept in order; otherwise W [k][n] -> B MN-major.
// OBF16: y is bf16 (round to nearest from the f32 accumulator) instead of f32.
// F16W: W is f16 ([k][n] or, with ROWS, [n][k]) instead of Q4; `scales` unused.
template <bool ROWS, bool OBF16, bool F16W>
__global__ void __launch_bounds__(kGmThreads, 1)
qm_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const uint8_t* __restrict__ packed,
               const uint16_t* __restrict__ scales, int T, int K, int N, void* __restrict__ y, int splits,
               float* __restrict__ partial, int* __restrict__ count, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    GmBars* bars = reinterpret_cast<GmBars*>(smem + kGmOffBar);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + kGmBN - 1) / kGmBN;
    // split-K: CTA (tile, split) takes k steps [kbeg, kbeg + nk) of the tile's K / 64
    const int tile = blockIdx.x / splits, split = blockIdx.x % splits;
    const int tm = tile / tiles_n, tn = tile % tiles_n;
    const int nk_all = K / kGmBK;
    const int kbeg = (int)((long long)split * nk_all / splits);
    const int nk = (int)((long long)(split + 1) * nk_all / splits) - kbeg;
    // a tile whose second 128 rows are all past T (a short prompt, or the last tile of one) loads,
    // multiplies and stores only its first half
    const bool two = tm * kGmBM + 128 < T;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGmStages; s++) {
            mbar_init(smem_u32(&bars->x_full[s]), 1);
            mbar_init(smem_u32(&bars->w_full[s]), kGmProdWarps);
            mbar_init(smem_u32(&bars->free_[s]), 1);
        }
        mbar_init(smem_u32(&bars->done), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kGmTmCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {  // X tiles by TMA
            prefetch_tmap(&tmx);
            int issued = 0;
            for (int i = 0; i < nk; i++) {
                const int s = i % kGmStages;
                if (i >= kGmStages &&
                    !mbar_wait_bounded(smem_u32(&bars->free_[s]), ((i / kGmStages) - 1) & 1, abort_flag, err)) {
                    *abort_flag = 1;
                    break;
                }
                const uint32_t xb = smem_u32(&bars->x_full[s]);
                mbar_arrive_expect_tx(xb, two ? 2 * kGmXBox : kGmXBox);
                const int kx = (kbeg + i) * kGmBK;
                tma_load_3d(sbase + s * kGmStage, &tmx, kx, tm * kGmBM, 0, xb);
                if (two) tma_load_3d(sbase + s * kGmStage + kGmXBox, &tmx, kx, tm * kGmBM + 128, 0, xb);
                issued = i + 1;
            }
            // every copy this thread issued has landed before the CTA can leave
            for (int i = issued - kGmStages > 0 ? issued - kGmStages : 0; i < issued; i++)
                mbar_drain(smem_u32(&bars->x_full[i % kGmStages]), (i / kGmStages) & 1, err);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issue
            bool ok = true;
            for (int i = 0; i < nk && ok; i++) {
                const int s = i % kGmStages;
                const uint32_t par = (i / kGmStages) & 1;
                ok = mbar_wait_bounded(smem_u32(&bars->x_full[s]), par, abort_flag, err) &&
                     mbar_wait_bounded(smem_u32(&bars->w_full[s]), par, abort_flag, err);
                if (!ok) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t xs = sbase + s * kGmStage, ws = xs + 2 * kGmXBox;
#pragma unroll
                for (int kk = 0; kk < kGmBK / 16; kk++) {  // one B, two A halves: rows 0-127, 128-255
                    const uint64_t bd = ROWS ? umma_sdesc(ws + kk * 32, 16, 1024) : umma_sdesc(ws + kk * 2048, kGmWBox, 1024);
                    const uint32_t id = ROWS ? kGmIdescRows : kGmIdesc;
                    umma_bf16_ss(tmem, umma_sdesc(xs + kk * 32, 16, 1024), bd, id, (i > 0 || kk > 0) ? 1u : 0u);
                    if (two)
                        umma_bf16_ss(tmem + kGmBN, umma_sdesc(xs + kGmXBox + kk * 32, 16, 1024), bd, id,
                                     (i > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(smem_u32(&bars->free_[s]));
            }
            umma_commit(smem_u32(&bars->done));  // every MMA issued above has completed
        }
    } else {  // warps 2..11: dequantise W tiles
        // thread pt takes chunks q = pt + 320 m of every stage; the words of the next two stages
        // are in flight while this stage's are converted
        const int pt = threadIdx.x - 64;  // 0..319
        const int n0_tile = tn * kGmBN;
        using WT = typename std::conditional<F16W, uint4, uint32_t>::type;  // one chunk's 8 weights
        WT wA[kGmChunks], wB[kGmChunks], wC[kGmChunks];
        uint16_t sA[kGmChunks], sB[kGmChunks], sC[kGmChunks];
        // per chunk m, fixed over the stages: the byte offset of its 4 nibble bytes (F16: 16
        // bytes) in stage 0 (a stage adds `stride`), for Q4 the scale at that offset >> 4 (the
        // chunk's place in its 32-group adds at most 12 bytes), its swizzled place in the stage's
        // B tile, and whether it is inside the tile (qmask) and inside W (okmask; outside, it
        // dequantises to zeros)
        uint32_t woff[kGmChunks], soff[kGmChunks], okmask = 0u, qmask = 0u;
#pragma unroll
        for (int m = 0; m < kGmChunks; m++) {
            const int q = pt + m * kGmProdWarps * 32;
            const bool inq = q < kGmBK * (kGmBN / 8);
            bool ok;
            if (ROWS) {  // row n = q / 8 of the tile, k chunk q % 8 (8 values: 4 bytes, one scale)
                const int n = n0_tile + (q >> 3);
                ok = inq && n < N;
                woff[m] = !ok ? 0u
                          : F16W ? (uint32_t)n * (uint32_t)(K * 2) + (uint32_t)(q & 7) * 16u
                                 : (uint32_t)n * (uint32_t)(K / 2) + (uint32_t)(q & 7) * 4u;
                soff[m] = sw128_off(q >> 3, q & 7);
            } else {  // k row q / 32 of the stage, 8 columns at (q % 32) * 8
                const int n0 = n0_tile + (q & 31) * 8;
                ok = inq && n0 < N;
                woff[m] = !ok ? 0u
                          : F16W ? (uint32_t)(q >> 5) * (uint32_t)(N * 2) + (uint32_t)(n0 * 2)
                                 : (uint32_t)(q >> 5) * (uint32_t)(N / 2) + (uint32_t)(n0 / 2);
                soff[m] = ((q & 31) >> 3) * kGmWBox + sw128_off(q >> 5, q & 7);
            }
            okmask |= (ok ? 1u : 0u) << m;
            qmask |= (inq ? 1u : 0u) << m;
        }
        const uint32_t stride = F16W ? (ROWS ? (uint32_t)(kGmBK * 2) : (uint32_t)kGmBK * (uint32_t)(N * 2))
                                     : (ROWS ? (uint32_t)(kGmBK / 2) : (uint32_t)kGmBK * (uint32_t)(N / 2));
        auto load_stage = [&](int i, WT(&wv)[kGmChunks], uint16_t(&sv)[kGmChunks]) {
            const uint32_t base = (uint32_t)(kbeg + i) * stride;
#pragma unroll
            for (int m = 0; m < kGmChunks; m++) {
                const bool ok = ((okmask >> m) & 1u) && i < nk;
                const uint32_t off = woff[m] + base;
                if constexpr (F16W) {
                    wv[m] = ok ? __ldg(reinterpret_cast<const uint4*>(packed + off)) : make_uint4(0u, 0u, 0u, 0u);
                } else {
                    wv[m] = ok ? __ldg(reinterpret_cast<const unsigned int*>(packed + off)) : 0x88888888u;
                    sv[m] = ok ? __ldg(reinterpret_cast<const unsigned short*>(scales + (off >> 4))) : (uint16_t)0;
                }
            }
        };
        // stage i into its ring slot (after the MMAs that read the slot last are done)
        auto convert_stage = [&](int i, const WT(&wv)[kGmChunks], const uint16_t(&sv)[kGmChunks]) -> bool {
            const int s = i % kGmStages;
            if (i >= kGmStages &&
                !mbar_wait_bounded(smem_u32(&bars->free_[s]), ((i / kGmStages) - 1) & 1, abort_flag, err)) {
                *abort_flag = 1;
                return false;
            }
            uint8_t* wt = smem + s * kGmStage + 2 * kGmXBox;
#pragma unroll
            for (int m = 0; m < kGmChunks; m++) {
                if (!((qmask >> m) & 1u)) break;
                if constexpr (F16W) {  // f16 pairs -> bf16 pairs (round to nearest), order kept
                    const uint32_t src[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w};
                    uint32_t pk[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const __nv_bfloat162 h =
                            __float22bfloat162_rn(__half22float2(*reinterpret_cast<const __half2*>(&src[j])));
                        pk[j] = *reinterpret_cast<const uint32_t*>(&h);
                    }
                    *reinterpret_cast<uint4*>(wt + soff[m]) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    continue;
                }
                // two nibbles per LOP3 as bf16x2 (128 + q, exact), minus 136 (exact), times the
                // scale in bf16: columns (c, c + 4) of the chunk land side by side, so the chunk's
                // 8 columns sit in the order 0 4 1 5 2 6 3 7 (the epilogue puts them back)
                const __nv_bfloat162 s2 = __float2bfloat162_rn(__half2float(__ushort_as_half(sv[m])));
                const __nv_bfloat162 c136 = __float2bfloat162_rn(136.0f);
                const uint32_t w = *reinterpret_cast<const uint32_t*>(&wv[m]);
                uint32_t pk[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t t = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
                    const __nv_bfloat162 h = __hmul2(__hsub2(*reinterpret_cast<const __nv_bfloat162*>(&t), c136), s2);
                    pk[j] = *reinterpret_cast<const uint32_t*>(&h);
                }
                if (ROWS)  // k must stay in order (it meets x's k): pairs (c, c+4) -> (c, c+1)
                    *reinterpret_cast<uint4*>(wt + soff[m]) =
                        make_uint4(__byte_perm(pk[0], pk[1], 0x5410), __byte_perm(pk[2], pk[3], 0x5410),
                                   __byte_perm(pk[0], pk[1], 0x7632), __byte_perm(pk[2], pk[3], 0x7632));
                else
                    *reinterpret_cast<uint4*>(wt + soff[m]) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars->w_full[s]));
            return true;
        };
        load_stage(0, wA, sA);
        load_stage(1, wB, sB);
        for (int i = 0; i < nk; i += 3) {  // three stages a turn: each buffer a fixed register set,
            load_stage(i + 2, wC, sC);     // loads two stages ahead of the conversion
            if (!convert_stage(i, wA, sA) || i + 1 >= nk) break;
            load_stage(i + 3, wA, sA);
            if (!convert_stage(i + 1, wB, sB) || i + 2 >= nk) break;
            load_stage(i + 4, wB, sB);
            if (!convert_stage(i + 2, wC, sC)) break;
        }
        if (warp >= 4 && warp < 8) {  // epilogue: TMEM lane quarter warp & 3
            const int quarter = warp & 3;
            const uint32_t la = (uint32_t)(quarter * 32) << 16;
            // 32 sums of row `row`, columns [col, col + 32), into y (rows past T and columns past N skipped)
            auto store32 = [&](int row, int col, const float* o) {
                if (row >= T || col >= N) return;
                if (!QM_IN((size_t)row * N + col, 32, (size_t)T * N, err)) return;
                if (OBF16) {
                    uint16_t* dst = static_cast<uint16_t*>(y) + (size_t)row * N + col;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        uint32_t h[4];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const __nv_bfloat162 b2 = __floats2bfloat162_rn(o[8 * q + 2 * e], o[8 * q + 2 * e + 1]);
                            h[e] = *reinterpret_cast<const uint32_t*>(&b2);
                        }
                        *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(h[0], h[1], h[2], h[3]);
                    }
                } else {
                    float* dst = static_cast<float*>(y) + (size_t)row * N + col;
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        *reinterpret_cast<float4*>(dst + 4 * q) = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
                }
            };
            if (mbar_wait_bounded(smem_u32(&bars->done), 0, abort_flag, err) && !*abort_flag) {
                tc_fence_after();
                // split-K: this CTA's partial tile as float4 [64 column quads][256 rows], so that the
                // lanes of a warp (consecutive rows) store and later load 512 contiguous bytes
                float4* mine = splits > 1 ? reinterpret_cast<float4*>(partial) + (size_t)blockIdx.x * (kGmBM * kGmBN / 4)
                                          : nullptr;
                for (int hf = 0; hf < (two ? 2 : 1); hf++) {  // accumulator hf: rows hf * 128 + lane quarter
                    const int r = hf * 128 + quarter * 32 + lane;
                    for (int c = 0; c < kGmBN / 32; c++) {
                        float v[32], o[32];
                        tmem_ld32(tmem + la + hf * kGmBN + c * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int p = 0; p < 32; p++)  // MN-major Q4 B: columns of each 8 in the order 0 4 1 5 2 6 3 7
                            o[(ROWS || F16W) ? p : (p & ~7) + ((p & 1) ? 4 : 0) + ((p & 7) >> 1)] = v[p];
                        if (splits == 1) {
                            store32(tm * kGmBM + r, n0_tile + c * 32, o);
                        } else if (QM_IN((size_t)blockIdx.x * (kGmBM * kGmBN / 4) + (c * 8 + 7) * kGmBM + r, 1,
                                         (size_t)gridDim.x * (kGmBM * kGmBN / 4), err)) {
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                __stcg(mine + (c * 8 + q) * kGmBM + r, make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]));
                        }
                    }
                }
            }
            if (splits > 1) {
                // every epilogue warp reaches both barriers on every path (an aborted CTA still counts
                // itself, so the tile's counter always returns to zero).  The counter update is a
                // release at GPU scope for the partial stores ordered before it by the barrier, and an
                // acquire: the last CTA then sees every split's partial.
                named_bar_sync(1, 128);
                if (warp == 4 && lane == 0) {
                    int prev = 0;
                    if (QM_IN(tile, 1, kSplitCounters, err))
                        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(count + tile)
                                     : "memory");
                    bars->last = prev == splits - 1;
                }
                named_bar_sync(1, 128);
                if (bars->last) {
                    if (!*abort_flag) {
                        const float4* tp = reinterpret_cast<const float4*>(partial) +
                                           (size_t)tile * splits * (kGmBM * kGmBN / 4);
                        for (int hf = 0; hf < (two ? 2 : 1); hf++) {
                            const int r = hf * 128 + quarter * 32 + lane;
                            for (int c = 0; c < kGmBN / 32; c++) {
                                float o[32];
#pragma unroll
                                for (int p = 0; p < 32; p++) o[p] = 0.f;
#pragma unroll
                                for (int sp = 0; sp < kGmMaxSplits; sp++) {  // in split order: the sum does not
                                    if (sp >= splits) break;                  // depend on timing
#pragma unroll
                                    for (int q = 0; q < 8; q++) {
                                        const size_t pi = (size_t)tile * splits * (kGmBM * kGmBN / 4) +
                                                          (sp * 64 + c * 8 + q) * kGmBM + r;
                                        const float4 f = QM_IN(pi, 1, (size_t)gridDim.x * (kGmBM * kGmBN / 4), err)
                                                             ? __ldcg(tp + ((sp * 64 + c * 8 + q) * kGmBM + r))
                                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                                        o[4 * q] += f.x;
                                        o[4 * q + 1] += f.y;
                                        o[4 * q + 2] += f.z;
                                        o[4 * q + 3] += f.w;
                                    }
                                }
                                store32(tm * kGmBM + r, n0_tile + c * 32, o);
                            }
                        }
                    }
                    if (warp == 4 && lane == 0 && QM_IN(tile, 1, kSplitCounters, err))
                        count[tile] = 0;  // ready for the next launch
                }
            }
        }
    }
    // the MMA thread committed `done` on every path: once it completes, no
    // MMA still writes TMEM
    if (warp == 1 && lane == 0) mbar_drain(smem_u32(&bars->done), 0, err);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kGmTmCols);
    }
}

}  // namespace
}  // namespace qm

using namespace qm;

static int gemm_call(qm_ctx* c, const qm_weight* w, int T, const uint16_t* x, void* y, bool obf16) {
    if (!c) return QM_E_ARG;
    if (!w || !x || !y || !w->data || T < 1 || w->k < 1 || w->n < 1)
        return set_error(c, QM_E_ARG, "null pointer or empty shape");
    const bool rows = w->kind == QM_W_Q4_ROWS || w->kind == QM_W_F16_ROWS;
    const bool f16w = w->kind == QM_W_F16 || w->kind == QM_W_F16_ROWS;
    if (w->kind != QM_W_Q4 && w->kind != QM_W_Q4_ROWS && !f16w)
        return set_error(c, QM_E_UNSUPPORTED, "qm_gemm takes QM_W_F16, QM_W_Q4, QM_W_F16_ROWS or QM_W_Q4_ROWS weights");
    if (!f16w && !w->scales) return set_error(c, QM_E_ARG, "Q4 weights need scales");
    if (w->k % kGmBK || w->n % 32) return set_error(c, QM_E_SHAPE, "qm_gemm needs k % 64 == 0 and n % 32 == 0");
    if ((uint64_t)w->k * (uint64_t)w->n * (f16w ? 2u : 1u) / (f16w ? 1u : 2u) >= (1ull << 32))
        return set_error(c, QM_E_SHAPE, "qm_gemm weights must be under 4 GB");
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 15) || ((uintptr_t)w->data & (f16w ? 15 : 3)) ||
        (!f16w && ((uintptr_t)w->scales & 1)))
        return set_error(c, QM_E_ARG, "x, y and F16 data must be 16-byte, Q4 data 4-byte and scales 2-byte aligned");
    cudaSetDevice(c->device);
    CUtensorMap tmx;
    if (encode_rows_tmap(&tmx, const_cast<uint16_t*>(x), (uint64_t)w->k, (uint64_t)T, 1, 64, 128, false) != QM_OK)
        return set_error(c, QM_E_CUDA, "cuTensorMapEncodeTiled failed for x");
    using Kern = void (*)(CUtensorMap, const uint8_t*, const uint16_t*, int, int, int, void*, int, float*, int*, int*);
    static const Kern kerns[8] = {
        qm_gemm_kernel<false, false, false>, qm_gemm_kernel<false, true, false>,
        qm_gemm_kernel<true, false, false>,  qm_gemm_kernel<true, true, false>,
        qm_gemm_kernel<false, false, true>,  qm_gemm_kernel<false, true, true>,
        qm_gemm_kernel<true, false, true>,   qm_gemm_kernel<true, true, true>};
    static std::atomic<uint64_t> attr_set[8];
    const int which = (f16w ? 4 : 0) + (rows ? 2 : 0) + (obf16 ? 1 : 0);
    const Kern kern = kerns[which];
    const uint64_t bit = 1ull << (c->device & 63);
    if (!(attr_set[which].load() & bit)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGmSmem);
        if (e != cudaSuccess) return cuda_error(c, e, "qm_gemm setup");
        attr_set[which].fetch_or(bit);
    }
    const int tiles = ((T + kGmBM - 1) / kGmBM) * ((w->n + kGmBN - 1) / kGmBN);
    // split K while the tiles would leave more than half the SMs idle: at most 4 splits, at least
    // 4 k-steps (256 of K) each, and no more CTAs than SMs (one CTA fills an SM)
    int splits = 1;
    if (2 * tiles <= c->num_sms) {
        splits = c->num_sms / tiles;
        splits = splits < kGmMaxSplits ? splits : kGmMaxSplits;
        splits = splits < w->k / (4 * kGmBK) ? splits : w->k / (4 * kGmBK);
        splits = splits > 1 ? splits : 1;
    }
    if (splits > 1) {
        const int rc = ensure_gemv_scratch(c, (size_t)tiles * splits * kGmBM * kGmBN * sizeof(float));
        if (rc != QM_OK) return rc;
    }
    TimedLaunch tl(c, "gemm");
    kern<<<tiles * splits, kGmThreads, kGmSmem, c->stream>>>(
        tmx, static_cast<const uint8_t*>(w->data), static_cast<const uint16_t*>(w->scales), T, w->k, w->n, y, splits,
        splits > 1 ? static_cast<float*>(c->gemv_partial) : nullptr, splits > 1 ? c->gemv_count : nullptr, c->d_err);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(c, e, "qm_gemm launch");
    c->launches += 1;
    return QM_OK;
}

extern "C" int qm_gemm(qm_ctx* c, const qm_weight* w, int T, const uint16_t* x, float* y) {
    return gemm_call(c, w, T, x, y, false);
}

extern "C" int qm_gemm_bf16(qm_ctx* c, const qm_weight* w, int T, const uint16_t* x, uint16_t* y) {
    return gemm_call(c, w, T, x, y, true);
}
