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
// Kernel: persistent, one CTA per SM walking 128 x 256 output tiles; warp 0
// lane 0 drives TMA (no multicast) through a 4-stage ring of 48 KB stages
// across tiles, warp 1 lane 0 issues tcgen05.mma (M=128, N=256, K=16, bf16 ->
// fp32 in TMEM) into one of two 256-column accumulators, and warps 2-5 drain the
// other with tcgen05.ld and store it, so a tile's epilogue overlaps the next
// tile's MMAs.  Every wait is bounded.
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
constexpr int TC_EPI0 = 2, TC_EPI_WARPS = 4;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int TC_THREADS = (TC_EPI0 + TC_EPI_WARPS) * 32;
constexpr uint32_t TC_TMEM_COLS = 2 * TC_BN;  // two accumulators: one fills while one drains
constexpr size_t TC_SMEM = (size_t)TC_STAGES * TC_STAGE_BYTES + 1024 + 256;

// kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1),
// B bf16 (bits 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22,
// M >> 4 at bits 24-28.
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                              ((uint32_t)(TC_BM >> 4) << 24);

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_bf16x3_kernel(const __grid_constant__ CUtensorMap mapA,
                       const __grid_constant__ CUtensorMap mapB, float* __restrict__ S,
                       int64_t lds, int M, int N, int nk, int m_fast, int* err) {
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * TC_STAGE_BYTES);
    uint64_t* empty = full + TC_STAGES;
    uint64_t* accfull = empty + TC_STAGES;  // 2: a tile's accumulator is complete
    uint64_t* accempty = accfull + 2;       // 2: the epilogue has drained it
    uint64_t* drain = accempty + 2;         // 1: every MMA issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mt = (M + TC_BM - 1) / TC_BM, nt = (N + TC_BN - 1) / TC_BN;
    const int64_t ntiles = mt * nt;
    // tile t -> (row tile, column tile); consecutive tiles share the larger
    // operand's tile while they walk the smaller operand, which stays in L2
    auto tile_of = [&](int64_t t, int* m0, int* n0) {
        const int64_t mi = m_fast ? t % mt : t / nt;
        const int64_t ni = m_fast ? t / mt : t % nt;
        *m0 = (int)(mi * TC_BM);
        *n0 = (int)(ni * TC_BN);
    };

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
        for (int s = 0; s < 2; ++s) {
            mbar_init(&accfull[s], 1);
            mbar_init(&accempty[s], TC_EPI_WARPS);
        }
        mbar_init(drain, 1);
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

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: every k-step of every tile of this CTA through the ring
        int64_t it = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            int m0, n0;
            tile_of(t, &m0, &n0);
            for (int kt = 0; kt < nk; ++kt, ++it) {
                const int s = (int)(it % TC_STAGES);
                if (it >= TC_STAGES &&
                    !mbar_wait(&empty[s], (uint32_t)((it / TC_STAGES) - 1) & 1u, err)) {
                    ok = false;
                    break;
                }
                unsigned char* sa = smem + s * TC_STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], TC_STAGE_BYTES);
                tma_load_2d(sa, &mapA, kt * TC_BK, m0, &full[s]);
                tma_load_2d(sa + TC_A_BYTES, &mapB, kt * TC_BK, n0, &full[s]);
            }
        }
        // no copy may still be landing when the CTA leaves
        for (int64_t k = it > TC_STAGES ? it - TC_STAGES : 0; k < it; ++k)
            mbar_drain(&full[k % TC_STAGES], (uint32_t)(k / TC_STAGES) & 1u);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: tile i accumulates in TMEM half i & 1 while the
        // epilogue drains the other half
        int64_t it = 0, lt = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++lt) {
            const int h = (int)(lt & 1);
            if (lt >= 2 && !mbar_wait(&accempty[h], (uint32_t)((lt >> 1) - 1) & 1u, err)) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(h * TC_BN);
            for (int kt = 0; kt < nk; ++kt, ++it) {
                const int s = (int)(it % TC_STAGES);
                if (!mbar_wait(&full[s], (uint32_t)(it / TC_STAGES) & 1u, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * TC_STAGE_BYTES);
                const uint32_t sb = sa + TC_A_BYTES;
#pragma unroll
                for (int k = 0; k < TC_BK / 16; ++k)
                    tc_mma_f16(d, sw128_desc(sa + k * 32), sw128_desc(sb + k * 32), TC_IDESC,
                               (kt | k) != 0);
                tc_commit(&empty[s]);  // frees the stage once these MMAs have read it
            }
            if (ok) tc_commit(&accfull[h]);
        }
        // fires once every MMA issued above has completed (also on an error path)
        tc_commit(drain);
        mbar_drain(drain, 0);
    } else if (warp >= TC_EPI0) {
        // ---- epilogue: warp w drains TMEM lanes 32 (w % 4) .. (= the tile's rows)
        const int quarter = warp & 3;
        int64_t lt = 0;
        for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
            const int h = (int)(lt & 1);
            if (!__all_sync(0xffffffffu, mbar_wait(&accfull[h], (uint32_t)(lt >> 1) & 1u, err))) break;
            tc_fence_after();
            int m0, n0;
            tile_of(t, &m0, &n0);
            const int row = m0 + quarter * 32 + lane;
            float* srow = S + (int64_t)row * lds;
#pragma unroll 1
            for (int c0 = 0; c0 < TC_BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(h * TC_BN + c0), r);
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[h]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
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

// One block per query row: the fp64 norm of its first d values (nrm_up >= ||x||
// rounded up, nrm2 ~ ||x||^2) and, with q3, its [hi | hi | lo] bf16 operand row
// (dims < dpad, zero padded to kp) -- the row norms and the query split in one
// read of the row.  Four dims per thread (16-byte loads, 8-byte stores) when the
// rows are 16-byte aligned, else one.
__device__ __forceinline__ uint32_t bf16_pair(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(128) query_prep_kernel(const float* __restrict__ X, int64_t ld,
                                                         int d, int dpad, int kp, int vec,
                                                         __nv_bfloat16* __restrict__ q3,
                                                         float* __restrict__ nrm_up,
                                                         float* __restrict__ nrm2) {
    __shared__ double part[4];
    const int64_t row = blockIdx.x;
    const float* x = X + row * ld;
    __nv_bfloat16* o = q3 ? q3 + row * (int64_t)kp : nullptr;
    double acc = 0.0;
    if (vec) {
        for (int i = 4 * threadIdx.x; i < dpad; i += 4 * blockDim.x) {
            const float4 v = *reinterpret_cast<const float4*>(x + i);
            const float xv[4] = {v.x, v.y, v.z, v.w};
            float lo[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (i + u < d) acc = fma((double)xv[u], (double)xv[u], acc);
                lo[u] = xv[u] - __bfloat162float(__float2bfloat16_rn(xv[u]));
            }
            if (o) {
                const uint2 hi = make_uint2(bf16_pair(xv[0], xv[1]), bf16_pair(xv[2], xv[3]));
                *reinterpret_cast<uint2*>(o + i) = hi;
                *reinterpret_cast<uint2*>(o + dpad + i) = hi;
                *reinterpret_cast<uint2*>(o + 2 * dpad + i) =
                    make_uint2(bf16_pair(lo[0], lo[1]), bf16_pair(lo[2], lo[3]));
            }
        }
    } else {
        for (int i = threadIdx.x; i < dpad; i += blockDim.x) {
            const float xv = x[i];
            if (i < d) acc = fma((double)xv, (double)xv, acc);
            if (o) {
                const __nv_bfloat16 hi = __float2bfloat16_rn(xv);
                o[i] = hi;
                o[dpad + i] = hi;
                o[2 * dpad + i] = __float2bfloat16_rn(xv - __bfloat162float(hi));
            }
        }
    }
    if (o)
        for (int j = 3 * dpad + threadIdx.x; j < kp; j += blockDim.x) o[j] = __float2bfloat16_rn(0.f);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        const double t = (part[0] + part[1]) + (part[2] + part[3]);
        if (nrm_up) nrm_up[row] = __double2float_ru(sqrt(t) * (1.0 + 1e-12));
        if (nrm2) nrm2[row] = (float)t;
    }
}

}  // namespace

cudaError_t launch_query_prep(const float* X, int64_t ld, int64_t n, int d, int dpad, int kp,
                              __nv_bfloat16* q3, float* nrm_up, float* nrm2, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    if (n > INT32_MAX) return cudaErrorInvalidValue;
    // 16-byte rows: every row start and dpad a multiple of 4 floats (then the
    // split row's segments start on 8-byte boundaries too, kp being a multiple of 64)
    const int vec = (ld % 4 == 0 && dpad % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(q3) & 7u) == 0 && kp % 4 == 0)
                        ? 1
                        : 0;
    query_prep_kernel<<<(unsigned)n, 128, 0, st>>>(X, ld, d, dpad, kp, vec, q3, nrm_up, nrm2);
    return cudaGetLastError();
}

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
    if (kp % TC_BK != 0) return cudaErrorInvalidValue;
    const int64_t mt = (M + TC_BM - 1) / TC_BM, nt = (N + TC_BN - 1) / TC_BN;
    // walk the smaller operand fastest: the A rows (M) when the B side is larger
    const int m_fast = N > M ? 1 : 0;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || sms <= 0) sms = 148;
    }
    cudaError_t e = cudaFuncSetAttribute(gemm_bf16x3_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)std::min<int64_t>(mt * nt, sms);
    gemm_bf16x3_kernel<<<grid, TC_THREADS, TC_SMEM, st>>>(mapA, mapB, S, lds, M, N, kp / TC_BK,
                                                          m_fast, err);
    return cudaGetLastError();
}

}  // namespace m3g
