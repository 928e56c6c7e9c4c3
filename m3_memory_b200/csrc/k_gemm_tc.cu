// k_gemm_tc.cu -- the coarse quantizer's query x centroid inner products on the
// 5th-generation tensor cores (tcgen05 + TMEM, operands staged by TMA).
//
// Accuracy: each fp32 value x is split into bf16 parts x = hi + lo + r with
// hi = bf16(x), lo = bf16(x - hi), |r| <= 2^-16 |x|.  The product a.b is taken as
// a_hi.b_hi + a_hi.b_lo + a_lo.b_hi (the bf16x3 scheme), written as one GEMM
// over K' = 3 D: A' = [a_hi | a_hi | a_lo], B' = [b_hi | b_lo | b_hi].  Per
// product the representation error is <= 3.02 * 2^-16 |a b|; the fp32
// accumulation of 3D terms is bounded without assuming the hardware's adder
// order (3D * 2^-23 of the sum of |terms|).  gemm_tc_error_beta() returns the
// resulting bound factor, which the exact selection (k_coarse.cu) relies on.
//
// Kernel: one CTA per 128 x 256 output tile; warp 0 lane 0 drives TMA (no
// multicast) through a 4-stage ring of 48 KB stages, warp 1 lane 0 issues
// tcgen05.mma (M=128, N=256, K=16, bf16 -> fp32 in TMEM, 256 columns), and all
// four warps drain TMEM with tcgen05.ld in the epilogue.  Every wait is bounded.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace m3g {
namespace {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64;  // bf16 elements; 64 x 2 B = 128 B rows
constexpr int TC_STAGES = 4;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;  // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;  // 32 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_THREADS = 128;
constexpr uint32_t TC_TMEM_COLS = 256;
constexpr size_t TC_SMEM = (size_t)TC_STAGES * TC_STAGE_BYTES + 1024 + 256;

// kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1),
// B bf16 (bits 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22,
// M >> 4 at bits 24-28.
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                              ((uint32_t)(TC_BM >> 4) << 24);

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_bf16x3_kernel(const __grid_constant__ CUtensorMap mapA,
                       const __grid_constant__ CUtensorMap mapB, float* __restrict__ S,
                       int64_t lds, int M, int N, int nk, int* err) {
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE_BYTES);
    uint64_t* empty = full + TC_STAGES;
    uint64_t* done = empty + TC_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * TC_BM, n0 = blockIdx.x * TC_BN;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (threadIdx.x == 0) {
        prefetch_tensormap(&mapA);
        prefetch_tensormap(&mapB);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = 0;  // TMA stages issued (producer lane)
    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        bool pok = true;
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % TC_STAGES;
            if (kt >= TC_STAGES && !mbar_wait(&empty[s], ((kt / TC_STAGES) - 1) & 1, err)) {
                pok = false;
                break;
            }
            unsigned char* sa = smem + s * TC_STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], TC_STAGE_BYTES);
            tma_load_2d(sa, &mapA, kt * TC_BK, m0, &full[s]);
            tma_load_2d(sa + TC_A_BYTES, &mapB, kt * TC_BK, n0, &full[s]);
            issued = kt + 1;
        }
        if (!pok) {  // error path: let the copies in flight land before leaving
            for (int kt = issued > TC_STAGES ? issued - TC_STAGES : 0; kt < issued; ++kt)
                mbar_drain(&full[kt % TC_STAGES], (kt / TC_STAGES) & 1);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer (one thread)
        for (int kt = 0; kt < nk; ++kt) {
            const int s = kt % TC_STAGES;
            if (!mbar_wait(&full[s], (kt / TC_STAGES) & 1, err)) break;
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * TC_STAGE_BYTES);
            const uint32_t sb = sa + TC_A_BYTES;
#pragma unroll
            for (int k = 0; k < TC_BK / 16; ++k)
                tc_mma_f16(tmem, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), TC_IDESC,
                       (kt | k) != 0);
            tc_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        // fires once every MMA issued above has completed (also on an error path)
        tc_commit(done);
    }

    // ---- epilogue: warp w owns TMEM lanes 32w .. 32w+31 (= output rows)
    __syncwarp();
    bool ok = mbar_wait(done, 0, err);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
        tc_fence_after();
        const int row = m0 + warp * 32 + lane;
        float* srow = S + (int64_t)row * lds;
#pragma unroll 1
        for (int c0 = 0; c0 < TC_BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
            if (row < M) {
                const int col = n0 + c0;
                if (col + 32 <= N && (lds & 3) == 0) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(srow + col + j) =
                            make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                        __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (col + j < N) srow[col + j] = __uint_as_float(r[j]);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // error path: the MMAs that were issued still complete into TMEM; wait
        // for them (bounded) before TMEM is released below
        mbar_drain(done, 0);
    } else if (warp == 0 && lane == 0) {
        // error path: no TMA copy may still be landing when the CTA leaves
        for (int kt = issued > TC_STAGES ? issued - TC_STAGES : 0; kt < issued; ++kt)
            mbar_drain(&full[kt % TC_STAGES], (kt / TC_STAGES) & 1);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TC_TMEM_COLS)
                     : "memory");
    }
}

// [hi | hi | lo] (queries) or [hi | lo | hi] (centroids), zero padded to kp.
__global__ void split3_kernel(const float* __restrict__ X, int64_t ld, int64_t n, int dpad, int kp,
                              __nv_bfloat16* __restrict__ out, int centroid_side) {
    const int64_t row = blockIdx.y;
    if (row >= n) return;
    const float* x = X + row * ld;
    __nv_bfloat16* o = out + row * (int64_t)kp;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < kp; j += gridDim.x * blockDim.x) {
        __nv_bfloat16 v = __float2bfloat16_rn(0.f);
        if (j < 3 * dpad) {
            const int seg = j / dpad, d = j - seg * dpad;
            const float xv = x[d];
            const __nv_bfloat16 hi = __float2bfloat16_rn(xv);
            const bool want_lo = centroid_side ? (seg == 1) : (seg == 2);
            v = want_lo ? __float2bfloat16_rn(xv - __bfloat162float(hi)) : hi;
        }
        o[j] = v;
    }
}

}  // namespace

int gemm_tc_kdim(int dpad) { return ((3 * dpad + TC_BK - 1) / TC_BK) * TC_BK; }

float gemm_tc_error_beta(int dpad) {
    // representation: 3.02 * 2^-16; accumulation: 3 dpad terms * 2^-23 * 1.008
    const double rep = 3.02 * 1.52587890625e-05;
    const double acc = 3.0 * (double)dpad * 1.1920928955078125e-07 * 1.008;
    return (float)((rep + acc) * 1.01);
}

int gemm_tc_box_rows_a() { return TC_BM; }
int gemm_tc_box_rows_b() { return TC_BN; }
int gemm_tc_box_k() { return TC_BK; }

cudaError_t launch_split3(const float* X, int64_t ld, int64_t n, int dpad, int kp,
                          __nv_bfloat16* out, bool centroid_side, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    for (int64_t b = 0; b < n; b += 65535) {
        const int64_t m = std::min<int64_t>(65535, n - b);
        dim3 grid((kp + 255) / 256, (unsigned)m);
        split3_kernel<<<grid, 256, 0, st>>>(X + b * ld, ld, m, dpad, kp, out + b * kp,
                                            centroid_side ? 1 : 0);
    }
    return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const CUtensorMap& mapA, const CUtensorMap& mapB, float* S, int64_t lds,
                           int M, int N, int kp, int* err, cudaStream_t st) {
    if (M <= 0 || N <= 0) return cudaSuccess;
    if (kp % TC_BK != 0 || M > 65535 * TC_BM) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16x3_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
    if (e != cudaSuccess) return e;
    dim3 grid((N + TC_BN - 1) / TC_BN, (M + TC_BM - 1) / TC_BM);
    gemm_bf16x3_kernel<<<grid, TC_THREADS, TC_SMEM, st>>>(mapA, mapB, S, lds, M, N, kp / TC_BK,
                                                          err);
    return cudaGetLastError();
}

}  // namespace m3g
