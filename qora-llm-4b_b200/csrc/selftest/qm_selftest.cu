// Test-only library (libqora_selftest.so, not part of the product library):
// a self-test of the tcgen05 / TMA building blocks the tensor-core kernels
// use — shared-memory and instruction descriptors, the 128-byte swizzle,
// operand A read from TMEM, MN-major B — on one tile against products the
// test computes in float64.  Links against libqora_mixer.so for the tensor
// map encoder.
#include <cuda_bf16.h>

#include "qm_internal.h"
#include "qm_ptx.cuh"

namespace qm {

int encode_rows_tmap(CUtensorMap* m, void* base, uint64_t inner, uint64_t rows, uint64_t planes,
                     uint32_t box_inner, uint32_t box_rows, bool fp16);

namespace {

constexpr int kBM = 128;                  // rows of A and P (UMMA M)
constexpr int kQBox = kBM * 128;          // [128 rows x 64 dims] 16-bit = 16 KB
constexpr int kTmQ = 0;                   // A copied into TMEM: 128 columns of 16-bit pairs
constexpr int kTmO = 256;                 // D2 accumulator, 256 columns
constexpr int kTmCols = 512;
constexpr uint32_t kIdescO = umma_idesc_f16kind(kBM, 256, false, true, false);

// Self-test layout (umma_selftest_kernel): one 64-key tile of each operand.
constexpr int kStKBox = 64 * 128;                 // [64 rows x 64 dims] = 8 KB
constexpr int kStOffQ = 0;
constexpr int kStOffK = kStOffQ + 4 * kQBox;
constexpr int kStOffV = kStOffK + 4 * kStKBox;
constexpr int kStOffP = kStOffV + 4 * kStKBox;
constexpr int kStOffBar = kStOffP + kBM * 128;
constexpr int kStSmem = kStOffBar + 256 + 1024;
constexpr int kStTmS = 128;
constexpr uint32_t kStIdescS = umma_idesc_f16kind(kBM, 64, false, false, false);
constexpr uint32_t kStIdescS_bf = umma_idesc_bf16(kBM, 64, false, false);
constexpr uint32_t kStIdescO_bf = umma_idesc_bf16(kBM, 256, false, true);
struct StBars {
    uint64_t ld_full, mma_done;
    uint32_t tmem_base;
    int abort_flag;
};


// Rows of a [128 x 256] 16-bit tile held as 4 TMA boxes of [128 rows x 64]
// (128-byte swizzle) -> TMEM, column col0 + d/2 of lane `row` holding dims d
// and d+1 (the A-operand layout of tcgen05.mma).
__device__ __forceinline__ void tile_rows_to_tmem(const uint8_t* tile, uint32_t taddr, int row) {
    for (int bx = 0; bx < 4; bx++) {
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
// Self-test of the tcgen05 building blocks (descriptors, TMEM mapping):
//   D1[128x64]  = A[128x256] . B[64x256]^T   (K-major A and B, TMA SW128; with
//                 mode bit 1 A is first copied to TMEM and read from there)
//   D2[128x256] = P[128x64]  . V[64x256]      (P written by threads, V MN-major)
// One CTA of 192 threads; the same descriptor and TMEM forms the prefill
// kernels use.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(192, 1)
umma_selftest_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                     const __grid_constant__ CUtensorMap tmv, const uint16_t* __restrict__ P,
                     float* __restrict__ d1, float* __restrict__ d2, int mode, int* err) {
    const bool fp16 = (mode & 1) != 0, a_tmem = (mode & 2) != 0;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    StBars* bars = reinterpret_cast<StBars*>(smem + kStOffBar);
    volatile int* abort_flag = &bars->abort_flag;
    const uint32_t sbase = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bars->ld_full), 1);
        mbar_init(smem_u32(&bars->mma_done), 1);
        bars->abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmCols);
        tmem_relinquish();
    }
    // P by plain stores into the swizzled K-major layout (rows of 64 bf16)
    for (int i = threadIdx.x; i < kBM * 8; i += blockDim.x) {
        const int row = i / 8, c = i % 8;
        const uint4 v = *reinterpret_cast<const uint4*>(P + row * 64 + c * 8);
        *reinterpret_cast<uint4*>(smem + kStOffP + sw128_off(row, c)) = v;
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = bars->tmem_base;
    const uint32_t qb = smem_u32(&bars->ld_full);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(qb, 4 * kQBox + 8 * kStKBox);
        for (int sub = 0; sub < 4; sub++) {
            tma_load_3d(sbase + kStOffQ + sub * kQBox, &tma, sub * 64, 0, 0, qb);
            tma_load_3d(sbase + kStOffK + sub * kStKBox, &tmb, sub * 64, 0, 0, qb);
            tma_load_3d(sbase + kStOffV + sub * kStKBox, &tmv, sub * 64, 0, 0, qb);
        }
    }
    bool ok = mbar_wait_bounded(qb, 0, abort_flag, err);
    if (ok && a_tmem && warp >= 2) {  // warps 2..5 own lane quarters 2, 3, 0, 1
        const int quarter = warp & 3;
        tile_rows_to_tmem(smem + kStOffQ, tm + ((uint32_t)(quarter * 32) << 16) + kTmQ, quarter * 32 + lane);
        tmem_st_wait();
    }
    tc_fence_before();
    ok = __syncthreads_and(ok) != 0;
    if (threadIdx.x == 0 && ok) {
        tc_fence_after();
        for (int kk = 0; kk < 16; kk++) {
            const uint64_t bd = umma_sdesc(sbase + kStOffK + (kk >> 2) * kStKBox + (kk & 3) * 32, 16, 1024);
            if (a_tmem)
                umma_f16_ts(tm + kStTmS, tm + kTmQ + kk * 8, bd, fp16 ? kStIdescS : kStIdescS_bf, kk > 0);
            else
                umma_bf16_ss(tm + kStTmS,
                             umma_sdesc(sbase + kStOffQ + (kk >> 2) * kQBox + (kk & 3) * 32, 16, 1024), bd,
                             fp16 ? kStIdescS : kStIdescS_bf, kk > 0);
        }
        for (int kk = 0; kk < 4; kk++)
            umma_bf16_ss(tm + kTmO, umma_sdesc(sbase + kStOffP + kk * 32, 16, 1024),
                         umma_sdesc(sbase + kStOffV + kk * 2048, kStKBox, 1024),
                         fp16 ? kIdescO : kStIdescO_bf, kk > 0);
        umma_commit(smem_u32(&bars->mma_done));
    }
    if (warp >= 2 && ok) {
        const int quarter = warp & 3, r = quarter * 32 + lane;
        const uint32_t la = (uint32_t)(quarter * 32) << 16;
        if (mbar_wait_bounded(smem_u32(&bars->mma_done), 0, abort_flag, err)) {
            tc_fence_after();
            for (int c = 0; c < 2; c++) {
                float v[32];
                tmem_ld32(tm + la + kStTmS + c * 32, v);
                tmem_ld_wait();
                for (int i = 0; i < 32; i++) d1[r * 64 + c * 32 + i] = v[i];
            }
            for (int c = 0; c < 8; c++) {
                float v[32];
                tmem_ld32(tm + la + kTmO + c * 32, v);
                tmem_ld_wait();
                for (int i = 0; i < 32; i++) d2[r * 256 + c * 32 + i] = v[i];
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


// Failure detection without a fault: 64 threads wait on an mbarrier nothing
// arrives at, through the library's bounded wait with a short limit.  The
// first thread to give up sets the error word and the CTA abort flag; the
// others then return at once.  Records how many waits succeeded (none
// should) and the longest wait in cycles.
__global__ void wait_timeout_selftest_kernel(long long limit, int* err, int* n_true, long long* max_cycles) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag_s;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag_s = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const long long t0 = clock64();
    const bool ok = mbar_wait_bounded(smem_u32(&bar), 0, &abort_flag_s, err, limit);
    const long long dt = clock64() - t0;
    if (ok) atomicAdd(n_true, 1);
    atomicMax(reinterpret_cast<unsigned long long*>(max_cycles), (unsigned long long)dt);
}

}  // namespace
}  // namespace qm

using namespace qm;

// Runs wait_timeout_selftest_kernel with `limit` cycles; returns the error
// word, the number of waits that succeeded and the longest wait.  The kernel
// ends normally either way: a QM status other than QM_OK means the launch
// itself failed.
extern "C" int qm_selftest_wait_timeout(long long limit, int* err_word, int* n_true, long long* max_cycles) {
    int* d = nullptr;
    if (cudaMalloc(&d, 4 * sizeof(long long)) != cudaSuccess) return QM_E_OOM;
    cudaMemset(d, 0, 4 * sizeof(long long));
    int* d_err = d;
    int* d_n = d + 2;
    long long* d_max = reinterpret_cast<long long*>(d) + 2;
    wait_timeout_selftest_kernel<<<1, 64>>>(limit, d_err, d_n, d_max);
    cudaError_t e = cudaDeviceSynchronize();
    long long h[4] = {0, 0, 0, 0};
    cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(d);
    if (e != cudaSuccess) return QM_E_CUDA;
    const int* hi = reinterpret_cast<const int*>(h);
    *err_word = hi[0];
    *n_true = hi[2];
    *max_cycles = h[2];
    return QM_OK;
}

// a [128x256], b [64x256], v [64x256], p [128x64] (device; all bf16, or all
// fp16 when mode bit 0 is set; mode bit 1: the first product reads a from
// TMEM); d1 [128x64], d2 [128x256] f32.  Synchronous; returns a QM status.
extern "C" int qm_selftest_umma(const uint16_t* a, const uint16_t* b, const uint16_t* v,
                                const uint16_t* p, float* d1, float* d2, int mode) {
    CUtensorMap ta, tb, tv;
    const bool h = (mode & 1) != 0;
    if (encode_rows_tmap(&ta, (void*)a, 256, 128, 1, 64, 128, h) != QM_OK ||
        encode_rows_tmap(&tb, (void*)b, 256, 64, 1, 64, 64, h) != QM_OK ||
        encode_rows_tmap(&tv, (void*)v, 256, 64, 1, 64, 64, h) != QM_OK)
        return QM_E_CUDA;
    int* err = nullptr;
    if (cudaMalloc(&err, sizeof(int)) != cudaSuccess) return QM_E_OOM;
    cudaMemset(err, 0, sizeof(int));
    cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStSmem);
    umma_selftest_kernel<<<1, 192, kStSmem>>>(ta, tb, tv, p, d1, d2, mode, err);
    cudaError_t e = cudaDeviceSynchronize();
    int flag = 0;
    cudaMemcpy(&flag, err, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (e != cudaSuccess) return QM_E_CUDA;
    return flag ? QM_E_TIMEOUT : QM_OK;
}
