// Projections around the mixers: y[b] = x[b] . W for the reference's weight
// formats (src/gemv.rs:21-40, 286-300): W [k rows (input) x n cols (output)],
//   F16  W[k][n] as f16 (gemv_f16, src/gemv.rs:338-368),
//   Q4   packed nibbles [k][n/2] (even column in the low nibble, value q - 8)
//        and f16 scales [k][n/32], one per 32 columns of a row (gemv_q4,
//        src/gemv.rs:411-450; format src/convert.rs:437-467).
// At decode batch sizes these are weight streams: every weight byte is read
// once per call and the arithmetic is a few operations per weight, so the
// kernel is HBM-bound and runs on the CUDA cores.  At batch 1 one launch
// moves 1.5-18 MB, i.e. 0.2-3 us of HBM time, so what the design fights is
// the fixed cost of a launch (start-up, load latency, the reduction) and
// the per-warp instruction stream:
//  * one launch covers up to kGvJobs weights that share the input x (the
//    reference's in_proj_qkv / z / a / b, or q / k / v_proj: one x_norm);
//  * every CTA issues its first weight loads before it waits for the
//    preceding kernel of the stream (programmatic dependent launch: weights
//    do not depend on it, x does), and lets the next kernel start at once;
//  * the rows of a column tile are split over as many CTAs as fill the GPU
//    in one wave (2 CTAs per SM), however few tiles the weight has;
//  * every weight load is 16 bytes a lane, 256-512 contiguous bytes a row,
//    and each row stream keeps R rows in flight (a rolling register ring:
//    the slot of the row just used is refilled with the row R ahead).
//
// qm_gemv_kernel<Q4, BT>: CTA (tile, part) takes output columns [tile T,
// (tile+1) T) (T = 512 Q4, 256 F16) and rows [part rps, (part+1) rps).  Each
// half-warp is one row stream: stream s (of 16 in a CTA) takes rows s, s+16,
// ... of the slice, lane h of the half-warp the CPL columns [CPL h, CPL h +
// CPL) of the tile: 16 bytes of nibbles (Q4: 32 columns, exactly one scale
// group) or 32 bytes of f16 (16 columns) per row.  Partial sums: the two
// half-warps by shuffle, the 8 warps in shared memory, the CTAs of a tile
// through a global scratch area: each CTA stores its partial, and the last
// CTA of the tile to finish (a counter) adds them (each warp a contiguous
// eighth of the parts, then the warps in order) and writes y.  Every sum is
// in a fixed order: the result does not depend on timing.  BT <= 4 sequences per launch; larger batches run in groups of 4.
//
// Q4 nibble without a shift or a conversion: the nibble q at bit 4j of a
// 16-bit half of the word, masked in place and read as a float, is the
// denormal q 2^(4j - 149); times s x 2^(100 - 4j) (4 products a row) it is
// q s x 2^-49 exactly, whatever j.  The column's sum is scaled back by 2^49
// and the -8 of every nibble enters once as -8 sum(s x) over the lane's rows
// (the same for its 32 columns).  One AND and one FFMA per weight at batch 1.
// (Valid while |s x| < 2^27; denormals are not flushed: no fast math.)
#include <cuda_fp16.h>

#include <atomic>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {
namespace {

constexpr int kGvWarps = 8;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvMaxParts = 64;
constexpr int kGvMaxB = 4;
constexpr int kGvJobs = 4;         // weights per launch
constexpr int kGvMaxTiles = kSplitCounters;  // counters in the scratch area

template <bool Q4>
struct GvShape {
    static constexpr int cpl = Q4 ? 32 : 16;  // columns per lane
    static constexpr int tile = 16 * cpl;     // columns per CTA
    static constexpr int pad = cpl + 4;       // shared-memory stride of a lane's columns
};

// rows in flight per stream (Q4 takes 5 registers a row, F16 8; at most what
// fits 2 CTAs per SM without spills).  Measured at batch 1 over the 32 layers'
// projections: Q4 6 rows 0.467 ms, 8 rows 0.472, 10-12 rows 0.489; F16 8 rows
// 0.552, 6 rows 0.559, 12 rows 0.569
template <bool Q4, int BT>
struct GvDepth {
    static constexpr int rows = BT == 1 ? (Q4 ? 6 : 8) : (BT == 2 ? 6 : 4);
};

struct GvJob {
    const void* data;
    const uint16_t* scales;
    float* y;  // [BT][n]
    int n;
    int tile0;  // first tile of this weight in the launch
};

struct GvArgs {
    GvJob job[kGvJobs];
    int njobs;
    int k;
    int parts;  // CTAs per tile
    int rows_per_part;
    const float* x;  // [BT][k]
    float* partial;  // [tiles][parts][BT][T] when parts > 1
    int* count;      // [tiles], zero between launches
};

template <bool Q4, int BT>
__global__ void __launch_bounds__(kGvThreads, BT <= 2 ? 2 : 1)
qm_gemv_kernel(const __grid_constant__ GvArgs a) {
    constexpr int R = GvDepth<Q4, BT>::rows, CPL = GvShape<Q4>::cpl, T = GvShape<Q4>::tile;
    constexpr int PAD = GvShape<Q4>::pad;
    constexpr int CPT = T / kGvThreads;  // columns per thread in the CTA sum
    extern __shared__ float smem_f[];
    __shared__ int last_cta;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int stream = warp * 2 + (lane >> 4), h = lane & 15;
    const int tile = blockIdx.x / a.parts, part = blockIdx.x % a.parts;
    int j = 0;
#pragma unroll
    for (int q = 1; q < kGvJobs; q++)
        if (q < a.njobs && tile >= a.job[q].tile0) j = q;
    const GvJob& jb = a.job[j];
    const int n = jb.n, k = a.k, rps = a.rows_per_part;
    const int r0 = part * rps;
    const int nr = max(0, min(k, r0 + rps) - r0);
    const int nrs = nr > stream ? (nr - stream + 15) / 16 : 0;  // rows of this stream
    float* xs = smem_f;                        // [BT][rps]
    float* red = xs + ((BT * rps + 3) & ~3);  // 16-byte aligned: [warps][BT][16 lanes][PAD]
    const int c0 = (tile - jb.tile0) * T + h * CPL;  // first of this lane's columns
    const bool live = c0 < n;
    const bool live2 = Q4 || c0 + 8 < n;  // F16: the lane's second 16 bytes (n % 16 may be 8)

    pdl_launch_dependents();
    uint4 wv[R][Q4 ? 1 : 2];
    uint32_t sv[Q4 ? R : 1];
    // row i of this stream (row stream + 16 i of the slice) into ring slot u
    auto load_row = [&](int u, int i) {
        const bool ok = live && i < nrs;
        const size_t row = (size_t)(r0 + stream + 16 * i);
        if (Q4) {
            const uint8_t* pk = static_cast<const uint8_t*>(jb.data);
            wv[u][0] = ok ? __ldcs(reinterpret_cast<const uint4*>(pk + row * (n / 2) + c0 / 2))
                          : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
            sv[u] = ok ? __ldcs(reinterpret_cast<const unsigned short*>(jb.scales + row * (n / 32) + c0 / 32)) : 0u;
        } else {
            const uint16_t* w16 = static_cast<const uint16_t*>(jb.data) + row * n + c0;
            wv[u][0] = ok ? __ldcs(reinterpret_cast<const uint4*>(w16)) : make_uint4(0u, 0u, 0u, 0u);
            wv[u][Q4 ? 0 : 1] = (ok && live2) ? __ldcs(reinterpret_cast<const uint4*>(w16 + 8))
                                              : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    // the first R rows: issued before waiting for the previous kernel
#pragma unroll
    for (int u = 0; u < R; u++) load_row(u, u);

    pdl_wait();  // x is written by the preceding kernel
    for (int i = tid; i < BT * nr; i += kGvThreads) {
        const int b = i / nr, r = i % nr;
        xs[b * rps + r] = a.x[(size_t)b * k + r0 + r];
    }
    __syncthreads();

    float acc[BT][CPL];
    // Q4 at batch 1: the column sums as pairs for the packed f32x2 FMA (two
    // products per instruction, each rounded as by fmaf; larger batches keep
    // scalar sums, the pairs' register alignment would spill them)
    constexpr bool kPacked = Q4 && BT == 1;
    float2 acc2[BT][kPacked ? CPL / 2 : 1];
    float sxsum[BT];  // Q4: the lane's sum of s x over its rows (the -8 of every nibble)
#pragma unroll
    for (int b = 0; b < BT; b++) {
        sxsum[b] = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; i++) acc[b][i] = 0.f;
#pragma unroll
        for (int i = 0; i < (kPacked ? CPL / 2 : 1); i++) acc2[b][i] = make_float2(0.f, 0.f);
    }

    for (int base = 0; base < nrs; base += R) {
#pragma unroll
        for (int u = 0; u < R; u++) {
            const int i = base + u;
            if (i >= nrs) break;
            const int r = stream + 16 * i;
            if (Q4) {
                const float s = __half2float(__ushort_as_half((uint16_t)sv[u]));
                float sxj[BT][4];  // s x 2^(100 - 4 jn): times the denormal nibble, q s x 2^-49
#pragma unroll
                for (int b = 0; b < BT; b++) {
                    const float sx = s * xs[b * rps + r];
                    sxsum[b] += sx;
#pragma unroll
                    for (int jn = 0; jn < 4; jn++) sxj[b][jn] = sx * (1.2676506e30f / (float)(1u << (4 * jn)));
                }
                const uint32_t ww[4] = {wv[u][0].x, wv[u][0].y, wv[u][0].z, wv[u][0].w};
                if (i + R < nrs) load_row(u, i + R);  // the slot's registers are copied: refill it
#pragma unroll
                for (int wd = 0; wd < 4; wd++) {
                    const uint32_t halves[2] = {ww[wd], ww[wd] >> 16};
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        // nibble 4 hh + jn of word wd (column 8 wd + 4 hh + jn of the lane's
                        // 32) masked in place: the denormal q 2^(4 jn - 149)
                        const uint32_t h = halves[hh];
                        if constexpr (kPacked) {  // two columns an instruction
                            const int c2 = 4 * wd + 2 * hh;
                            acc2[0][c2] = __ffma2_rn(make_float2(__uint_as_float(h & 0xFu), __uint_as_float(h & 0xF0u)),
                                                     make_float2(sxj[0][0], sxj[0][1]), acc2[0][c2]);
                            acc2[0][c2 + 1] =
                                __ffma2_rn(make_float2(__uint_as_float(h & 0xF00u), __uint_as_float(h & 0xF000u)),
                                           make_float2(sxj[0][2], sxj[0][3]), acc2[0][c2 + 1]);
                        } else {
#pragma unroll
                            for (int jn = 0; jn < 4; jn++) {
                                const float v = __uint_as_float(h & (0xFu << (4 * jn)));
#pragma unroll
                                for (int b = 0; b < BT; b++)
                                    acc[b][8 * wd + 4 * hh + jn] = fmaf(v, sxj[b][jn], acc[b][8 * wd + 4 * hh + jn]);
                            }
                        }
                    }
                }
            } else {
                float xv[BT];
#pragma unroll
                for (int b = 0; b < BT; b++) xv[b] = xs[b * rps + r];
                const uint4 w0 = wv[u][0], w1 = wv[u][Q4 ? 0 : 1];
                if (i + R < nrs) load_row(u, i + R);
                const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[q]));
#pragma unroll
                    for (int b = 0; b < BT; b++) {
                        acc[b][2 * q] = fmaf(xv[b], f.x, acc[b][2 * q]);
                        acc[b][2 * q + 1] = fmaf(xv[b], f.y, acc[b][2 * q + 1]);
                    }
                }
            }
        }
    }
    if constexpr (kPacked) {
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int i = 0; i < CPL / 2; i++) {
                acc[b][2 * i] = acc2[b][i].x;
                acc[b][2 * i + 1] = acc2[b][i].y;
            }
    }
    // the two half-warps (same columns, other rows), then the 8 warps, each in
    // a fixed order
#pragma unroll
    for (int b = 0; b < BT; b++)
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            if (Q4) acc[b][i] = fmaf(acc[b][i], 562949953421312.0f, -8.0f * sxsum[b]);  // 2^49 sum q s x - 8 sum s x
            acc[b][i] += __shfl_xor_sync(0xffffffffu, acc[b][i], 16);
        }
    if (lane < 16) {
#pragma unroll
        for (int b = 0; b < BT; b++)
#pragma unroll
            for (int q = 0; q < CPL / 4; q++)
                *reinterpret_cast<float4*>(&red[((warp * BT + b) * 16 + h) * PAD + 4 * q]) =
                    make_float4(acc[b][4 * q], acc[b][4 * q + 1], acc[b][4 * q + 2], acc[b][4 * q + 3]);
    }
    __syncthreads();
    float psum[BT][CPT];
#pragma unroll
    for (int b = 0; b < BT; b++)
#pragma unroll
        for (int c = 0; c < CPT; c++) {
            const int col = c * kGvThreads + tid;
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < kGvWarps; w++) sum += red[((w * BT + b) * 16 + col / CPL) * PAD + col % CPL];
            psum[b][c] = sum;
        }
    const int tcol = (tile - jb.tile0) * T;
    if (a.parts == 1) {
#pragma unroll
        for (int c = 0; c < CPT; c++)
            if (tcol + c * kGvThreads + tid < n)
#pragma unroll
                for (int b = 0; b < BT; b++) jb.y[(size_t)b * n + tcol + c * kGvThreads + tid] = psum[b][c];
        return;
    }
    // the CTAs of the tile: store this partial; the last CTA to finish adds
    // them.  Thread 0's counter update is a release at GPU scope (after the
    // barrier it orders the whole CTA's stores) and an acquire (the last CTA
    // then sees every other CTA's partial): no separate fences.
    float* mine = a.partial + ((size_t)blockIdx.x * BT) * T;
#pragma unroll
    for (int b = 0; b < BT; b++)
#pragma unroll
        for (int c = 0; c < CPT; c++) __stcg(&mine[b * T + c * kGvThreads + tid], psum[b][c]);
    __syncthreads();
    if (tid == 0) {
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(a.count + tile) : "memory");
        last_cta = prev == a.parts - 1;
    }
    __syncthreads();
    if (!last_cta) return;
    // The last CTA's sum is spread over its warps so that few L2 round trips
    // are in series: warp w adds the contiguous parts [w P/8, (w+1) P/8) of all
    // T columns (lane: LC columns as float4s, the loads of 4 parts in flight),
    // then the 8 warp sums are added in warp order through shared memory (the
    // CTA-sum area, no longer read).  A fixed order: the result does not depend
    // on which CTA finished last.
    const float* tp = a.partial + ((size_t)tile * a.parts * BT) * T;
    constexpr int LC = T / 32;  // columns per lane: 16 Q4, 8 F16
    float* wsum = red;          // [warps][BT][T]; fits the [warps][BT][16][PAD] area
    const int pw0 = (a.parts * warp) / kGvWarps, pw1 = (a.parts * (warp + 1)) / kGvWarps;
#pragma unroll
    for (int b = 0; b < BT; b++) {
        float4 s[LC / 4];
#pragma unroll
        for (int q = 0; q < LC / 4; q++) s[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = pw0; p < pw1; p += 4) {
            float4 v[4][LC / 4];
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int q = 0; q < LC / 4; q++)
                    v[u][q] = p + u < pw1 ? __ldcg(reinterpret_cast<const float4*>(
                                                tp + ((size_t)(p + u) * BT + b) * T + lane * LC) + q)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (p + u < pw1)
#pragma unroll
                    for (int q = 0; q < LC / 4; q++) {
                        s[q].x += v[u][q].x;
                        s[q].y += v[u][q].y;
                        s[q].z += v[u][q].z;
                        s[q].w += v[u][q].w;
                    }
        }
#pragma unroll
        for (int q = 0; q < LC / 4; q++)
            *reinterpret_cast<float4*>(&wsum[((size_t)warp * BT + b) * T + lane * LC + 4 * q]) = s[q];
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < BT; b++)
#pragma unroll
        for (int c = 0; c < CPT; c++) {
            const int col = c * kGvThreads + tid;
            float tot = 0.f;
#pragma unroll
            for (int w = 0; w < kGvWarps; w++) tot += wsum[((size_t)w * BT + b) * T + col];
            if (tcol + col < n) jb.y[(size_t)b * n + tcol + col] = tot;
        }
    if (tid == 0) a.count[tile] = 0;  // ready for the next launch
}

size_t gemv_smem(bool q4, int bt, int rps) {
    const int pad = q4 ? GvShape<true>::pad : GvShape<false>::pad;
    return (size_t)(((bt * rps + 3) & ~3) + kGvWarps * bt * 16 * pad) * 4;
}
int gemv_tile(bool q4) { return q4 ? GvShape<true>::tile : GvShape<false>::tile; }

// Per device and kernel instantiation: the shared-memory attribute is set
// once, and how many CTAs fit on an SM (registers are what limit this kernel).
struct GvOccupancy {
    std::atomic<int> ready{0};
    int per_sm = 1;
};

template <bool Q4, int BT>
cudaError_t gemv_setup(qm_ctx* ctx, GvOccupancy** out) {
    static GvOccupancy occ[64];
    GvOccupancy& o = occ[ctx->device & 63];
    *out = &o;
    if (o.ready.load()) return cudaSuccess;
    auto kern = qm_gemv_kernel<Q4, BT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kGvThreads, gemv_smem(Q4, BT, 256));
    if (e != cudaSuccess) return e;
    o.per_sm = nb > 0 ? nb : 1;
    o.ready.store(1);
    return cudaSuccess;
}

template <bool Q4, int BT>
cudaError_t launch_bt(qm_ctx* ctx, GvArgs& a, int tiles) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * a.parts);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = gemv_smem(Q4, BT, a.rows_per_part);
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qm_gemv_kernel<Q4, BT>, a);
}

template <bool Q4>
cudaError_t launch_kind(qm_ctx* ctx, GvArgs& a, int bt, int tiles) {
    switch (bt) {
        case 1: return launch_bt<Q4, 1>(ctx, a, tiles);
        case 2: return launch_bt<Q4, 2>(ctx, a, tiles);
        case 3: return launch_bt<Q4, 3>(ctx, a, tiles);
        default: return launch_bt<Q4, 4>(ctx, a, tiles);
    }
}

template <bool Q4>
cudaError_t setup_kind(qm_ctx* ctx, int bt, GvOccupancy** o) {
    switch (bt) {
        case 1: return gemv_setup<Q4, 1>(ctx, o);
        case 2: return gemv_setup<Q4, 2>(ctx, o);
        case 3: return gemv_setup<Q4, 3>(ctx, o);
        default: return gemv_setup<Q4, 4>(ctx, o);
    }
}

// CTAs per tile: as many as keep the launch to one wave, at least 16 rows each.
int pick_parts(const qm_ctx* c, const GvOccupancy& o, int tiles, int k) {
    int p = o.per_sm * c->num_sms / tiles;
    p = p < k / 16 ? p : k / 16;
    p = p < kGvMaxParts ? p : kGvMaxParts;
    return p > 1 ? p : 1;
}

}  // namespace

int ensure_gemv_scratch(qm_ctx* c, size_t partial_bytes) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    const bool capturing = cudaStreamIsCapturing(c->stream, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone;
    if ((!c->gemv_count || partial_bytes > c->gemv_partial_bytes) && capturing)
        return set_error(c, QM_E_CAPTURE, "qm_gemv scratch must grow during stream capture; call it once first");
    if (!c->gemv_count) {
        if (cudaMalloc(&c->gemv_count, kGvMaxTiles * sizeof(int)) != cudaSuccess) {
            c->gemv_count = nullptr;
            return set_error(c, QM_E_OOM, "qm_gemv: scratch counters");
        }
        QM_CHECK_CUDA(c, cudaMemsetAsync(c->gemv_count, 0, kGvMaxTiles * sizeof(int), c->stream));
    }
    if (partial_bytes <= c->gemv_partial_bytes) return QM_OK;
    QM_CHECK_CUDA(c, cudaStreamSynchronize(c->stream));
    if (c->gemv_partial) cudaFree(c->gemv_partial);
    c->gemv_partial = nullptr;
    c->gemv_partial_bytes = 0;
    if (cudaMalloc(&c->gemv_partial, partial_bytes) != cudaSuccess) {
        c->gemv_partial = nullptr;
        return set_error(c, QM_E_OOM, "qm_gemv: scratch partials");
    }
    c->gemv_partial_bytes = partial_bytes;
    return QM_OK;
}

}  // namespace qm

using namespace qm;

extern "C" int qm_gemv_multi(qm_ctx* c, const qm_weight* ws, int count, int batch, const float* x,
                             float* const* ys) {
    if (!c) return QM_E_ARG;
    if (!ws || !x || !ys || count < 1 || batch < 1) return set_error(c, QM_E_ARG, "null pointer or empty batch");
    if (count > kGvJobs) return set_error(c, QM_E_SHAPE, "at most 4 weights per call");
    const int k = ws[0].k, kind = ws[0].kind;
    if (kind == QM_W_F16_ROWS || kind == QM_W_Q4_ROWS) {  // one row per output: the lm_head kernel
        if (count != 1) return set_error(c, QM_E_SHAPE, "row-layout weights take one weight per call");
        if (!ws[0].data || !ys[0] || ws[0].k < 1 || ws[0].n < 1)
            return set_error(c, QM_E_ARG, "null pointer or empty shape");
        return gemv_rows(c, &ws[0], batch, x, ys[0]);
    }
    const bool q4 = kind == QM_W_Q4;
    int tiles = 0;
    for (int i = 0; i < count; i++) {
        const qm_weight* w = &ws[i];
        if (!w->data || !ys[i] || w->k < 1 || w->n < 1) return set_error(c, QM_E_ARG, "null pointer or empty shape");
        if (w->k != k || w->kind != kind) return set_error(c, QM_E_MISMATCH, "weights of one call differ in k or kind");
        if (w->kind == QM_W_Q4) {
            if (!w->scales) return set_error(c, QM_E_ARG, "Q4 weights need scales");
            if (w->n % 32) return set_error(c, QM_E_SHAPE, "Q4 needs n % 32 == 0 (groups of 32)");
            if (((uintptr_t)w->data & 15) || ((uintptr_t)w->scales & 1))
                return set_error(c, QM_E_ARG, "Q4 data must be 16-byte and scales 2-byte aligned");
        } else if (w->kind == QM_W_F16) {
            if (w->n % 8) return set_error(c, QM_E_SHAPE, "F16 needs n % 8 == 0");
            if ((uintptr_t)w->data & 15) return set_error(c, QM_E_ARG, "F16 data must be 16-byte aligned");
        } else {
            return set_error(c, QM_E_ARG, "unknown weight kind");
        }
        tiles += (w->n + gemv_tile(q4) - 1) / gemv_tile(q4);
    }
    if (tiles > kGvMaxTiles) return set_error(c, QM_E_SHAPE, "too many output columns for one call");
    cudaSetDevice(c->device);
    const int bt0 = batch < kGvMaxB ? batch : kGvMaxB;  // the first launch's batch (the largest)
    GvOccupancy* occ = nullptr;
    cudaError_t se = q4 ? setup_kind<true>(c, bt0, &occ) : setup_kind<false>(c, bt0, &occ);
    if (se != cudaSuccess) return cuda_error(c, se, "qm_gemv setup");
    const int parts = pick_parts(c, *occ, tiles, k);
    const int rps = (k + parts - 1) / parts;
    if (gemv_smem(q4, kGvMaxB, rps) > 200 * 1024) return set_error(c, QM_E_SHAPE, "k too large for one CTA's rows");
    if (parts > 1) {
        const int rc = ensure_gemv_scratch(c, (size_t)tiles * parts * bt0 * gemv_tile(q4) * sizeof(float));
        if (rc != QM_OK) return rc;
    }
    TimedLaunch tl(c, "gemv");
    GvArgs a = {};
    a.njobs = count;
    a.k = k;
    a.parts = parts;
    a.rows_per_part = rps;
    a.partial = static_cast<float*>(c->gemv_partial);
    a.count = c->gemv_count;
    for (int b0 = 0; b0 < batch; b0 += kGvMaxB) {
        const int bt = batch - b0 < kGvMaxB ? batch - b0 : kGvMaxB;
        int t0 = 0;
        for (int i = 0; i < count; i++) {
            a.job[i].data = ws[i].data;
            a.job[i].scales = static_cast<const uint16_t*>(ws[i].scales);
            a.job[i].y = ys[i] + (size_t)b0 * ws[i].n;
            a.job[i].n = ws[i].n;
            a.job[i].tile0 = t0;
            t0 += (ws[i].n + gemv_tile(q4) - 1) / gemv_tile(q4);
        }
        a.x = x + (size_t)b0 * k;
        if (bt != bt0) {  // the last, smaller group: its instantiation's attributes
            GvOccupancy* o2 = nullptr;
            se = q4 ? setup_kind<true>(c, bt, &o2) : setup_kind<false>(c, bt, &o2);
            if (se != cudaSuccess) return cuda_error(c, se, "qm_gemv setup");
        }
        const cudaError_t e = q4 ? launch_kind<true>(c, a, bt, tiles) : launch_kind<false>(c, a, bt, tiles);
        if (e != cudaSuccess) return cuda_error(c, e, "qm_gemv launch");
        c->launches += 1;
    }
    return QM_OK;
}

extern "C" int qm_gemv(qm_ctx* c, const qm_weight* w, int batch, const float* x, float* y) {
    if (!c) return QM_E_ARG;
    if (!w) return set_error(c, QM_E_ARG, "null weight");
    return qm_gemv_multi(c, w, 1, batch, x, &y);
}
