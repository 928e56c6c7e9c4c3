// k_coarse.cu -- coarse quantizer: row norms, the approximate query x centroid
// inner-product matrix (SIMT fp32 variant; the tcgen05 variant lives in
// k_gemm_tc.cu), and the exact top-nprobe / nearest-centroid selection.
//
// Selection contract (IVFIndex::select_nprobe_for_query,
// AgentMemory/M3/src/m3_index.cpp:492-523, and IVFIndex::nearest_clusters,
// :243-264): for each query, the P centroids with the smallest unified score as
// the reference computes it (fp32, index-order sums, one rounding per op),
// ascending.  Exact ties go to the lower cluster id (the reference leaves them
// to nth_element / sort, or to its strict '<' scan, which is the same rule for
// P = 1).
//
// Method: the approximate scores come with a rigorous error bound e_c, so
// [a_c - e_c, a_c + e_c] holds the reference's value.  With T the P-th smallest
// upper bound, no centroid whose lower bound exceeds T can be among the P
// smallest.  The remaining candidates (normally P plus a handful) are rescored
// in the reference's exact arithmetic and sorted by (score, id).
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "score.cuh"

namespace m3g {

// ---------------------------------------------------------------------------
// Row norms: one warp per row, fp64 accumulation.  nrm_up[i] >= ||x_i|| (an
// upper bound rounded up to fp32), nrm2[i] ~ ||x_i||^2 in fp32.
// ---------------------------------------------------------------------------
__global__ void row_norms_kernel(const float* __restrict__ X, int64_t ld, int64_t n, int d,
                                 float* __restrict__ nrm_up, float* __restrict__ nrm2) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float* x = X + row * ld;
    double acc = 0.0;
    for (int i = lane; i < d; i += 32) {
        double v = (double)x[i];
        acc = fma(v, v, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        if (nrm_up) nrm_up[row] = __double2float_ru(sqrt(acc) * (1.0 + 1e-12));
        if (nrm2) nrm2[row] = (float)acc;
    }
}

void launch_row_norms(const float* X, int64_t ld, int64_t n, int d, float* nrm_up, float* nrm2,
                      cudaStream_t st) {
    if (n <= 0) return;
    const int rows_per_block = 8;
    const int64_t grid = (n + rows_per_block - 1) / rows_per_block;
    row_norms_kernel<<<(unsigned)grid, rows_per_block * 32, 0, st>>>(X, ld, n, d, nrm_up, nrm2);
}

// ---------------------------------------------------------------------------
// SIMT fp32 GEMM, S[m][n] = sum_k A[m][k] * B[n][k] (both K-contiguous).
// 128x128 tile, BK = 8, 256 threads, 8x8 outputs per thread.  Error bound for
// any summation order with or without FMA: |S - exact| <= (K+2) 2^-24 sum|a b|.
// ---------------------------------------------------------------------------
namespace {
constexpr int GB_M = 128, GB_N = 128, GB_K = 8;
}

__global__ void __launch_bounds__(256) sgemm_nt_kernel(const float* __restrict__ A, int64_t lda,
                                                       const float* __restrict__ B, int64_t ldb,
                                                       float* __restrict__ S, int64_t lds, int M,
                                                       int N, int K) {
    __shared__ __align__(16) float As[2][GB_K][GB_M];
    __shared__ __align__(16) float Bs[2][GB_K][GB_N];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * GB_M, n0 = blockIdx.x * GB_N;
    // loader mapping: 128 rows x 8 k = 256 threads x float4
    const int lr = tid >> 1, lk = (tid & 1) * 4;
    const int tx = tid & 15, ty = tid >> 4;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    auto load = [&](int buf, int k0) {
        float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = make_float4(0.f, 0.f, 0.f, 0.f);
        const int ar = m0 + lr, br = n0 + lr, kk = k0 + lk;
        if (ar < M) {
            const float* p = A + (int64_t)ar * lda + kk;
            if (kk + 3 < K) va = *reinterpret_cast<const float4*>(p);
            else {
                if (kk < K) va.x = p[0];
                if (kk + 1 < K) va.y = p[1];
                if (kk + 2 < K) va.z = p[2];
            }
        }
        if (br < N) {
            const float* p = B + (int64_t)br * ldb + kk;
            if (kk + 3 < K) vb = *reinterpret_cast<const float4*>(p);
            else {
                if (kk < K) vb.x = p[0];
                if (kk + 1 < K) vb.y = p[1];
                if (kk + 2 < K) vb.z = p[2];
            }
        }
        As[buf][lk + 0][lr] = va.x;
        As[buf][lk + 1][lr] = va.y;
        As[buf][lk + 2][lr] = va.z;
        As[buf][lk + 3][lr] = va.w;
        Bs[buf][lk + 0][lr] = vb.x;
        Bs[buf][lk + 1][lr] = vb.y;
        Bs[buf][lk + 2][lr] = vb.z;
        Bs[buf][lk + 3][lr] = vb.w;
    };

    load(0, 0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += GB_K) {
        if (k0 + GB_K < K) load(buf ^ 1, k0 + GB_K);
#pragma unroll
        for (int kk = 0; kk < GB_K; ++kk) {
            float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
        buf ^= 1;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (c < N) S[(int64_t)r * lds + c] = acc[i][j];
        }
    }
}

void launch_sgemm_nt(const float* A, int64_t lda, const float* B, int64_t ldb, float* S,
                     int64_t lds, int M, int N, int K, cudaStream_t st) {
    if (M <= 0 || N <= 0) return;
    dim3 grid((N + GB_N - 1) / GB_N, (M + GB_M - 1) / GB_M);
    sgemm_nt_kernel<<<grid, 256, 0, st>>>(A, lda, B, ldb, S, lds, M, N, K);
}

float sgemm_error_beta(int K) { return (float)(K + 2) * 5.9604645e-8f * 1.01f; }

// ---------------------------------------------------------------------------
// GEMV for a few rows of A (tiny query batches): S[m][n] = sum_k A[m][k] B[n][k]
// for m < M <= GEMV_MAX_M.  A is staged in shared memory; each warp takes one row
// of B at a time with 16-byte loads along k, keeps the M dot products per lane
// and reduces them over the warp.  fp32 FMAs in another order than the GEMM's, so
// the same bound holds (sgemm_error_beta: any summation order, with or without
// FMA).  The whole grid streams B once, where the tiled GEMMs give a single
// row of A a few CTAs.
// ---------------------------------------------------------------------------
constexpr int GEMV_MAX_M = 8;
constexpr int GEMV_SMEM_MAX = 48 * 1024;

__global__ void __launch_bounds__(256) gemv_nt_kernel(const float* __restrict__ A, int64_t lda,
                                                      const float* __restrict__ B, int64_t ldb,
                                                      float* __restrict__ S, int64_t lds, int M,
                                                      int N, int K) {
    extern __shared__ __align__(16) float as[];  // [M][K]
    for (int i = threadIdx.x; i < M * K; i += blockDim.x) {
        const int m = i / K, k = i - m * K;
        as[i] = A[(int64_t)m * lda + k];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int k4n = K / 4;
    for (int n = blockIdx.x * nw + warp; n < N; n += gridDim.x * nw) {
        const float4* b = reinterpret_cast<const float4*>(B + (int64_t)n * ldb);
        float acc[GEMV_MAX_M];
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) acc[m] = 0.f;
        for (int k4 = lane; k4 < k4n; k4 += 32) {
            const float4 v = __ldg(b + k4);
#pragma unroll
            for (int m = 0; m < GEMV_MAX_M; ++m) {
                if (m < M) {
                    const float4 a = reinterpret_cast<const float4*>(as + m * K)[k4];
                    acc[m] = fmaf(a.x, v.x, acc[m]);
                    acc[m] = fmaf(a.y, v.y, acc[m]);
                    acc[m] = fmaf(a.z, v.z, acc[m]);
                    acc[m] = fmaf(a.w, v.w, acc[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < GEMV_MAX_M; ++m) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && m < M) S[(int64_t)m * lds + n] = v;
        }
    }
}

bool gemv_fits(const float* A, int64_t lda, const float* B, int64_t ldb, int M, int K) {
    return M >= 1 && M <= GEMV_MAX_M && K % 4 == 0 && ldb % 4 == 0 &&
           (reinterpret_cast<uintptr_t>(B) & 15u) == 0 && (size_t)M * K * 4 <= GEMV_SMEM_MAX;
}

void launch_gemv_nt(const float* A, int64_t lda, const float* B, int64_t ldb, float* S,
                    int64_t lds, int M, int N, int K, int num_sms, cudaStream_t st) {
    if (M <= 0 || N <= 0) return;
    const int blocks = (int)std::min<int64_t>((N + 7) / 8, (int64_t)num_sms * 8);
    gemv_nt_kernel<<<blocks, 256, (size_t)M * K * 4, st>>>(A, lda, B, ldb, S, lds, M, N, K);
}

// ---------------------------------------------------------------------------
// Exact selection.
// ---------------------------------------------------------------------------
namespace {
// Two shapes of the selection block: a small one (128 threads, 256 candidates,
// about 28 KB of shared memory for 4096 centroids of dim 1024, so that seven
// blocks share an SM and a batch of 1024 queries runs in one wave: every phase
// waits on memory, and more resident queries hide more of it) for P <= 128, and
// a large one (256 threads, 1024 candidates) for larger P.
constexpr int SEL_SMALL_NT = 128, SEL_SMALL_CAP = 256, SEL_SMALL_MINB = 7;
constexpr int SEL_LARGE_NT = 256, SEL_LARGE_CAP = 1024;
constexpr int SEL_SMALL_P = 128;     // largest P for the small block
constexpr int SEL_KEYS_SMEM = 8192;  // upper-bound keys cached in shared memory up to this L
constexpr int SEL_SORT_MAX = 1024;   // largest P whose selection is returned sorted
constexpr int SEL_OVERLAP_MAX = 128; // above this many candidates the overlap test sorts
constexpr int SEL_STAGE = kExactTileFloats;  // per-warp product tile of the exact rescoring
constexpr int SEL_KEEP_LO_L = 8192;  // largest L whose lower-bound keys stay beside S0
constexpr int SEL_UNROLL = 8;        // centroids per thread whose bounds load together
constexpr uint32_t kKeyNegInf = 0x007fffffu;  // float_key(-inf)
constexpr uint32_t kKeyPosInf = 0xff800000u;  // float_key(+inf)
static_assert(SEL_LARGE_CAP >= SEL_SORT_MAX && SEL_SMALL_CAP >= SEL_SMALL_P,
              "the sorted fallback keeps P keys in the candidate array");
static_assert(3 * SEL_SMALL_CAP <= (SEL_SMALL_NT / 32) * SEL_STAGE &&
                  3 * SEL_LARGE_CAP <= (SEL_LARGE_NT / 32) * SEL_STAGE,
              "S0 lives in the tile area");
static_assert(SEL_SMALL_P <= SEL_SMALL_NT, "the small block's P takes its pre-filtered path");

// 32-bit words of the shared area that holds, in turn, the cached upper-bound
// keys or the lower-bound keys beside S0, and the per-warp product tiles.
template <int NT, int CAP>
__host__ __device__ constexpr size_t sel_area_words(int L) {
    size_t a = (size_t)(NT / 32) * SEL_STAGE;
    if (L <= SEL_KEYS_SMEM && (size_t)L > a) a = (size_t)L;
    if (L <= SEL_KEEP_LO_L && (size_t)L + 3 * CAP > a) a = (size_t)L + 3 * CAP;
    return a;
}

template <int NT>
struct SelShared {
    unsigned hist[256];
    unsigned mins[NT / 32];
    unsigned prefix, remain, count, count2, m_less, tie_need, tkey, nex, nin, wtot[NT / 32];
};

// Finds the rank-th smallest (1-based) of the keys produced by key_of(c),
// c in [0, L), by 4 passes of an 8-bit radix select.  All threads return it.
template <int NT, class KeyOf>
__device__ uint32_t block_radix_select(KeyOf key_of, int L, unsigned rank, SelShared<NT>& sh) {
    uint32_t prefix = 0, mask = 0;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < 256; i += NT) sh.hist[i] = 0;
        __syncthreads();
        for (int c0 = 0; c0 < L; c0 += NT) {
            const int c = c0 + threadIdx.x;
            int bin = -1;
            if (c < L) {
                const uint32_t k = key_of(c);
                if ((k & mask) == prefix) bin = (int)((k >> shift) & 255u);
            }
            // near-equal keys share a bin: one atomic per distinct bin per warp
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (bin >= 0 && (threadIdx.x & 31) == __ffs(peers) - 1)
                atomicAdd(&sh.hist[bin], (unsigned)__popc(peers));
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // warp 0 scans the 256 bins: lane l owns bins 8l..8l+7
            unsigned loc[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                loc[j] = sh.hist[threadIdx.x * 8 + j];
                s += loc[j];
            }
            unsigned incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if ((int)threadIdx.x >= o) incl += v;
            }
            const unsigned excl = incl - s;
            if (excl < rank && rank <= incl) {
                unsigned r = rank - excl;
                int b = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (b == 0 && r <= loc[j]) b = j + 1;
                    else if (b == 0) r -= loc[j];
                }
                sh.prefix = prefix | ((uint32_t)(threadIdx.x * 8 + b - 1) << shift);
                sh.remain = r;
            }
        }
        __syncthreads();
        prefix = sh.prefix;
        rank = sh.remain;
        mask |= 255u << shift;
        __syncthreads();
    }
    return prefix;
}

// Block-wide exclusive scan of one flag per thread; returns the thread's offset
// and writes the block total to *total.
template <int NT>
__device__ unsigned block_flag_scan(bool flag, unsigned* total, SelShared<NT>& sh) {
    const unsigned lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const unsigned ball = __ballot_sync(0xffffffffu, flag);
    const unsigned below = __popc(ball & ((1u << lane) - 1u));
    if (lane == 0) sh.wtot[w] = __popc(ball);
    __syncthreads();
    unsigned base = 0, tot = 0;
    for (unsigned i = 0; i < NT / 32; ++i) {
        if (i < w) base += sh.wtot[i];
        tot += sh.wtot[i];
    }
    __syncthreads();
    *total = tot;
    return base + below;
}

// Bitonic sort of one key per lane, ascending across lanes.
__device__ __forceinline__ uint32_t warp_sort_asc_u32(uint32_t v, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint32_t p = __shfl_xor_sync(0xffffffffu, v, j);
            const bool up = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            v = (lower == up) ? (p < v ? p : v) : (p > v ? p : v);
        }
    }
    return v;
}

template <int NT>
__device__ void bitonic_sort_u64(unsigned long long* a, int n) {
    // n is a power of two
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += NT) {
                const int p = i ^ j;
                if (p > i) {
                    const unsigned long long x = a[i], y = a[p];
                    const bool up = (i & k) == 0;
                    if ((x > y) == up) {
                        a[i] = y;
                        a[p] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}
}  // namespace

// One block per query.  S holds the approximate inner products (overwritten
// with exact scores on the fallback path).  Writes P cluster ids per query into
// probes (ascending by exact score when P <= 1024, else in ascending id order),
// or -1 for the nearest-cluster form (P == 1, kSelectNanIsNone) when every score
// is NaN.  With kSelectSetOnly the row holds the same set of ids in an order of
// the kernel's choosing (deterministic), and only the candidates whose
// membership the intervals leave open are rescored exactly.
template <int NT, int CAP, int MINB>
__global__ void __launch_bounds__(NT, MINB) select_probes_kernel(
    float* __restrict__ S, int64_t lds, const float* __restrict__ Q, int64_t ldq,
    const float* __restrict__ C, int64_t ldc, const float* __restrict__ qn,
    const float* __restrict__ qn2, const float* __restrict__ cn, const float* __restrict__ cn2,
    int L, int D, int metric, int normalized, float beta, float gamma, int P, int flags,
    int32_t* __restrict__ probes) {
    extern __shared__ __align__(16) unsigned char sel_smem[];
    __shared__ SelShared<NT> sh;
    constexpr int NW = NT / 32;
    const int q = blockIdx.x;
    float* qs = reinterpret_cast<float*>(sel_smem);                               // D floats
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(qs + ((D + 3) & ~3));  // CAP
    float2* bnd = reinterpret_cast<float2*>(cand + CAP);                     // CAP
    int* exl = reinterpret_cast<int*>(bnd);  // reuses bnd once the overlap test is done
    unsigned char* needf = reinterpret_cast<unsigned char*>(bnd + CAP);      // CAP
    // one area, used first for the cached upper-bound keys, later for the
    // per-warp product tiles of the exact rescoring
    uint32_t* hkeys = reinterpret_cast<uint32_t*>(needf + CAP);
    float* stage_all = reinterpret_cast<float*>(hkeys);
    const bool cache = L <= SEL_KEYS_SMEM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool nan_is_none = (flags & kSelectNanIsNone) != 0;
    const bool set_only = (flags & kSelectSetOnly) != 0;

    const float* qrow = Q + (int64_t)q * ldq;
    for (int i = threadIdx.x; i < D; i += NT) qs[i] = qrow[i];
    float* srow = S + (int64_t)q * lds;
    const float nq = qn[q], nq2 = qn2[q];
    const bool nrm = normalized != 0;
    if (threadIdx.x == 0) {  // read after later barriers on every path
        sh.nex = 0;
        sh.nin = 0;
    }

    auto bounds = [&](int c, float* lo, float* hi) {
        approx_bounds(srow[c], nq, cn[c], nq2, cn2[c], beta, gamma, metric, nrm, lo, hi);
    };
    const int PP = P < L ? P : L;
    bool exact_all = PP > SEL_SORT_MAX;
    bool have = false;  // candidates in cand[0, cnt)
    unsigned cnt = 0;
    // interval of candidate i as keys (lower, upper), beside cand[i]
    uint2* ik = reinterpret_cast<uint2*>(bnd);
    // the pre-filtered threshold serves P up to 32 per warp (each warp offers its
    // ceil(P / NW)-th key): 128 in the small block, 256 in the large one
    if (!exact_all && PP <= 32 * NW) {
        // --- pre-filtered threshold.  Small block: each of the NW warps sorts its
        // threads' smallest upper-bound keys and offers its ceil(PP/NW)-th smallest;
        // tau0, the largest offer, has at least NW * ceil(PP/NW) >= PP distinct keys
        // <= it.  Larger P (over 32 in the small block, every P in the large one):
        // every thread keeps its TOPT smallest keys (2 / 4) and tau0 is the PP-th
        // smallest of those NT * TOPT keys (a far tighter threshold than the offers,
        // whose largest is the largest thread minimum).
        // Either way tau0 >= T (the PP-th smallest upper bound of all).  Every centroid with
        // hi <= T therefore has lo <= tau0, so T is the PP-th smallest upper bound
        // within S0 = {c : lo <= tau0}, and every candidate (lo <= T) is in S0.
        // The lower-bound keys of the first pass are kept when they fit beside S0.
        // Loops over centroids take SEL_UNROLL of them per thread at a time with
        // their loads issued together.
        uint32_t* lkeys = hkeys;
        const bool keep_lo = L <= SEL_KEEP_LO_L;  // the area then holds L + 3 CAP words
        constexpr int TOPT = NT == SEL_LARGE_NT ? 4 : 2;
        // small P in the small block: the warp offers (cheap, tight enough there)
        const bool offers = NT != SEL_LARGE_NT && PP <= 32;
        static_assert(TOPT * NT <= CAP, "the thread minima fit the S0 key array");
        uint32_t mk[TOPT];  // this thread's TOPT smallest upper-bound keys, ascending
#pragma unroll
        for (int j = 0; j < TOPT; ++j) mk[j] = 0xffffffffu;
        for (int c0 = threadIdx.x; c0 < L; c0 += SEL_UNROLL * NT) {
            float sv[SEL_UNROLL], av[SEL_UNROLL], bv[SEL_UNROLL];
#pragma unroll
            for (int u = 0; u < SEL_UNROLL; ++u) {
                const int c = c0 + u * NT;
                sv[u] = c < L ? srow[c] : 0.f;
                av[u] = c < L ? cn[c] : 0.f;
                bv[u] = c < L ? cn2[c] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < SEL_UNROLL; ++u) {
                const int c = c0 + u * NT;
                if (c < L) {
                    float lo, hi;
                    approx_bounds(sv[u], nq, av[u], nq2, bv[u], beta, gamma, metric, nrm, &lo, &hi);
                    uint32_t k = float_key(hi);
#pragma unroll
                    for (int j = 0; j < TOPT; ++j) {
                        const uint32_t m = mk[j];
                        mk[j] = k < m ? k : m;
                        k = k < m ? m : k;
                    }
                    if (keep_lo) lkeys[c] = lo != lo ? 0u : float_key(lo);
                }
            }
        }
        uint32_t* f_id = hkeys + (keep_lo ? L : 0);  // S0, in the key / tile area
        uint32_t* f_lo = f_id + CAP;
        uint32_t* f_hi = f_lo + CAP;
        if (offers) {
            const uint32_t sorted = warp_sort_asc_u32(mk[0], lane);
            const uint32_t offer = __shfl_sync(0xffffffffu, sorted, (PP + NW - 1) / NW - 1);
            if (lane == 0) sh.mins[warp] = offer;
        } else {
            // the pool of thread minima, in the S0 upper-bound array until S0 fills it
#pragma unroll
            for (int j = 0; j < TOPT; ++j) f_hi[threadIdx.x * TOPT + j] = mk[j];
        }
        if (threadIdx.x == 0) {
            sh.count = 0;
            sh.count2 = 0;
            sh.tkey = 0xffffffffu;
        }
        __syncthreads();
        uint32_t tau0 = 0;
        if (offers) {
            for (int w = 0; w < NW; ++w) tau0 = sh.mins[w] > tau0 ? sh.mins[w] : tau0;
        } else {
            // every key of the pool is a distinct centroid's, and the pool holds at
            // least min(L, NT * TOPT) >= PP real keys (a thread keeps all of its
            // keys when L <= NT * TOPT), so at least PP centroids have hi <= tau0
            tau0 = block_radix_select([&](int i) { return f_hi[i]; }, NT * TOPT, (unsigned)PP, sh);
        }
        auto s0_add = [&](int c, uint32_t lk) {
            if (lk <= tau0) {
                const unsigned slot = atomicAdd(&sh.count, 1u);
                if (slot < (unsigned)CAP) {
                    f_id[slot] = (uint32_t)c;
                    f_lo[slot] = lk;
                }
            }
        };
        if (keep_lo) {
            for (int c = threadIdx.x; c < L; c += NT) s0_add(c, lkeys[c]);
        } else {
            for (int c0 = threadIdx.x; c0 < L; c0 += SEL_UNROLL * NT) {
                float sv[SEL_UNROLL], av[SEL_UNROLL], bv[SEL_UNROLL];
#pragma unroll
                for (int u = 0; u < SEL_UNROLL; ++u) {
                    const int c = c0 + u * NT;
                    sv[u] = c < L ? srow[c] : 0.f;
                    av[u] = c < L ? cn[c] : 0.f;
                    bv[u] = c < L ? cn2[c] : 0.f;
                }
#pragma unroll
                for (int u = 0; u < SEL_UNROLL; ++u) {
                    const int c = c0 + u * NT;
                    if (c < L) {
                        float lo, hi;
                        approx_bounds(sv[u], nq, av[u], nq2, bv[u], beta, gamma, metric, nrm, &lo,
                                      &hi);
                        s0_add(c, lo != lo ? 0u : float_key(lo));
                    }
                }
            }
        }
        __syncthreads();
        const unsigned n0 = sh.count;
        if (n0 <= (unsigned)CAP) {
            // upper bounds of S0: few centroids, their loads in parallel
            for (int i = threadIdx.x; i < (int)n0; i += NT) {
                float lo, hi;
                bounds((int)f_id[i], &lo, &hi);
                f_hi[i] = float_key(hi);
            }
            __syncthreads();
            // T = the PP-th smallest upper bound in S0 (n0 >= PP, see above)
            uint32_t tkey;
            if (n0 <= (unsigned)NT) {
                // by counting: the one key value with fewer than PP keys below it
                // and at least PP at or below it
                if (threadIdx.x < n0) {
                    const uint32_t k = f_hi[threadIdx.x];
                    unsigned less = 0, le = 0;
                    for (int j = 0; j < (int)n0; ++j) {
                        const uint32_t kj = f_hi[j];
                        less += kj < k ? 1u : 0u;
                        le += kj <= k ? 1u : 0u;
                    }
                    if (less < (unsigned)PP && le >= (unsigned)PP) sh.tkey = k;
                }
                __syncthreads();
                tkey = sh.tkey;
            } else {
                tkey = block_radix_select([&](int i) { return f_hi[i]; }, (int)n0, (unsigned)PP, sh);
            }
            // candidates: lo <= T, with their intervals
            for (int i = threadIdx.x; i < (int)n0; i += NT) {
                if (f_lo[i] <= tkey) {
                    const unsigned slot = atomicAdd(&sh.count2, 1u);
                    cand[slot] = f_id[i];
                    ik[slot] = make_uint2(f_lo[i], f_hi[i]);
                }
            }
            __syncthreads();
            cnt = sh.count2;
            have = true;
        }
        // else S0 overflows: the general path below recomputes every bound
    }
    // T once the general path has it: the fallback then needs exact scores only for
    // the centroids whose lower bound is within it
    bool have_t = false;
    uint32_t t_all = 0xffffffffu;
    if (!exact_all && !have) {
        if (cache) {
            for (int c = threadIdx.x; c < L; c += NT) {
                float lo, hi;
                bounds(c, &lo, &hi);
                hkeys[c] = float_key(hi);
            }
        }
        __syncthreads();
        // --- phase A: T = PP-th smallest upper bound
        uint32_t tkey;
        if (cache)
            tkey = block_radix_select([&](int c) { return hkeys[c]; }, L, (unsigned)PP, sh);
        else
            tkey = block_radix_select(
                [&](int c) {
                    float lo, hi;
                    bounds(c, &lo, &hi);
                    return float_key(hi);
                },
                L, (unsigned)PP, sh);
        have_t = true;
        t_all = tkey;
        // --- phase B: candidates whose lower bound is <= T (compared as keys,
        // so a NaN bound, key 0xffffffff for hi / mapped low for lo, is kept)
        if (threadIdx.x == 0) sh.count = 0;
        __syncthreads();
        for (int c = threadIdx.x; c < L; c += NT) {
            float lo, hi;
            bounds(c, &lo, &hi);
            const uint32_t lk = lo != lo ? 0u : float_key(lo);
            if (lk <= tkey) {
                const unsigned slot = atomicAdd(&sh.count, 1u);
                if (slot < (unsigned)CAP) {
                    cand[slot] = (unsigned long long)c;
                    ik[slot] = make_uint2(lk, float_key(hi));
                }
            }
        }
        __syncthreads();
        cnt = sh.count;
        if (cnt > (unsigned)CAP) exact_all = true;
        else have = true;
    }
    if (have) {
        // --- phase C: order the candidates by exact score.  The intervals hold
        // the reference's scores, so a candidate whose finite interval overlaps no
        // other candidate's is ordered, against all others (their exact scores
        // included), by its lower bound; the rest are rescored in the reference's
        // exact arithmetic.  Keys: (score key, id), all distinct.
        //
        // Set mode needs only membership.  Candidate i is in for certain when
        // fewer than PP others can precede it (lower bound <= its upper bound):
        // then its upper bound is <= T, so no non-candidate (lower bound > T) can.
        // It is out for certain when PP others precede it for certain (upper
        // bound < its lower bound).  Only the rest are rescored (needf 1; 0 in,
        // 2 out), and the in-for-certain ones are ordered by their lower bounds.
        constexpr int PER = CAP / NT;  // candidates per thread in the pairwise loops
        static_assert(CAP % NT == 0, "whole candidates per thread");
        const bool set_mode = set_only && !nan_is_none;
        if (set_mode) {
            // PX candidates per thread (1 when they fit one per thread: the warps
            // past the last candidate then skip the loop)
            auto classify = [&](auto px) {
                constexpr int PX = decltype(px)::value;
                if ((int)threadIdx.x >= (int)cnt) return;
                uint2 bi[PX];
                unsigned maybe_before[PX], surely_before[PX];
#pragma unroll
                for (int u = 0; u < PX; ++u) {
                    const int i = threadIdx.x + u * NT;
                    bi[u] = i < (int)cnt ? ik[i] : make_uint2(0u, 0u);
                    maybe_before[u] = 0;
                    surely_before[u] = 0;
                }
                for (int j = 0; j < (int)cnt; ++j) {
                    const uint2 bj = ik[j];
#pragma unroll
                    for (int u = 0; u < PX; ++u) {
                        maybe_before[u] += bj.x <= bi[u].y ? 1u : 0u;
                        surely_before[u] += bj.y < bi[u].x ? 1u : 0u;
                    }
                }
#pragma unroll
                for (int u = 0; u < PX; ++u) {
                    const int i = threadIdx.x + u * NT;
                    if (i >= (int)cnt) continue;
                    // the loop counted the candidate against itself too
                    const unsigned mb = maybe_before[u] - (bi[u].x <= bi[u].y ? 1u : 0u);
                    const unsigned sb = surely_before[u] - (bi[u].y < bi[u].x ? 1u : 0u);
                    unsigned char st = 1;
                    if (bi[u].x > kKeyNegInf && bi[u].y < kKeyPosInf) {
                        if (mb < (unsigned)PP) st = 0;
                        else if (sb >= (unsigned)PP) st = 2;
                    }
                    if (st == 0) atomicAdd(&sh.nin, 1u);
                    needf[i] = st;
                }
            };
            if (cnt <= (unsigned)NT) classify(std::integral_constant<int, 1>{});
            else classify(std::integral_constant<int, PER>{});
        } else if (cnt <= (unsigned)SEL_OVERLAP_MAX) {
            // few candidates: every pair of intervals compared
            for (int i = threadIdx.x; i < (int)cnt; i += NT) {
                const uint2 bi = ik[i];
                bool need = bi.x <= kKeyNegInf || bi.y >= kKeyPosInf;
                for (int j = 0; j < (int)cnt && !need; ++j) {
                    const uint2 bj = ik[j];
                    if (j != i && bj.x <= bi.y && bi.x <= bj.y) need = true;
                }
                needf[i] = need ? 1 : 0;
            }
        } else {
            // many: in the order of the lower bounds (ties by position), a candidate
            // overlaps an earlier one iff the largest earlier upper bound reaches
            // its lower bound, and a later one iff the next lower bound is within
            // its upper bound.  Sort keys and the running maximum use the tile
            // area (free until the rescoring below).
            unsigned long long* srt = reinterpret_cast<unsigned long long*>(stage_all);  // CAP
            uint32_t* hmax = reinterpret_cast<uint32_t*>(srt + CAP);                     // CAP
            int n2 = 1;
            while (n2 < (int)cnt) n2 <<= 1;
            for (int i = threadIdx.x; i < n2; i += NT)
                srt[i] = i < (int)cnt ? (((unsigned long long)ik[i].x << 32) | (unsigned)i) : ~0ull;
            __syncthreads();
            bitonic_sort_u64<NT>(srt, n2);
            for (int p = threadIdx.x; p < (int)cnt; p += NT)
                hmax[p] = ik[(uint32_t)(srt[p] & 0xffffffffu)].y;
            __syncthreads();
            // inclusive running maximum of the upper bounds (Hillis-Steele)
            for (int d = 1; d < (int)cnt; d <<= 1) {
                uint32_t v[PER];
#pragma unroll
                for (int u = 0; u < PER; ++u) {
                    const int p = threadIdx.x + u * NT;
                    v[u] = 0;
                    if (p < (int)cnt) v[u] = p >= d ? max(hmax[p], hmax[p - d]) : hmax[p];
                }
                __syncthreads();
#pragma unroll
                for (int u = 0; u < PER; ++u) {
                    const int p = threadIdx.x + u * NT;
                    if (p < (int)cnt) hmax[p] = v[u];
                }
                __syncthreads();
            }
            for (int p = threadIdx.x; p < (int)cnt; p += NT) {
                const int i = (int)(srt[p] & 0xffffffffu);
                const uint2 bi = ik[i];
                bool need = bi.x <= kKeyNegInf || bi.y >= kKeyPosInf;
                if (p > 0 && hmax[p - 1] >= bi.x) need = true;
                if (p + 1 < (int)cnt && (uint32_t)(srt[p + 1] >> 32) <= bi.y) need = true;
                needf[i] = need ? 1 : 0;
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < (int)cnt; i += NT) {
            const unsigned c = (unsigned)cand[i];
            cand[i] = needf[i] == 1 ? (unsigned long long)c : ((unsigned long long)ik[i].x << 32) | c;
        }
        __syncthreads();
        // compact the candidates to rescore (exl reuses the interval array)
        for (int i = threadIdx.x; i < (int)cnt; i += NT)
            if (needf[i] == 1) exl[atomicAdd(&sh.nex, 1u)] = i;
        __syncthreads();
        const int nex = (int)sh.nex;
        float* stage = stage_all + warp * SEL_STAGE;
        for (int r0 = 0; r0 < nex; r0 += NT) {
            // up to NT candidates per round, G per warp.  With the blocks of a batch
            // resident in one wave the kernel's time is a block's latency, which
            // the shortest per-warp share and the widest chunks keep lowest; a
            // warp's time is set by its chunk width, not by how many of its lanes
            // hold candidates, so a warp takes up to 8 (the widest chunks) before
            // the next takes any, and the idle warps leave the SM's issue slots to
            // the blocks beside it.  More than 8 per warp: ceil(n / NW) each.
            const int n = nex - r0 < NT ? nex - r0 : NT;
            const int G = min(n, max(8, (n + NW - 1) / NW));
            if (warp * G >= n) continue;  // warp-uniform: nothing for this warp
            const int i = warp * G + lane;
            const int idx = (lane < G && i < n) ? exl[r0 + i] : -1;
            const int c = idx >= 0 ? (int)(cand[idx] & 0xffffffffu) : -1;
            float r;
            if (G <= 8)
                r = warp_exact_scores<4>(qs, C, ldc, D, metric, nrm, c, stage, lane);
            else if (G <= 16)
                r = warp_exact_scores<2>(qs, C, ldc, D, metric, nrm, c, stage, lane);
            else
                r = warp_exact_scores<1>(qs, C, ldc, D, metric, nrm, c, stage, lane);
            if (idx >= 0) cand[idx] = ((unsigned long long)float_key(r) << 32) | (unsigned)c;
        }
        __syncthreads();
        if (set_mode) {
            // positions: the nin in-for-certain ids by (lower-bound key, id), then
            // the best PP - nin rescored ones by (exact key, id)
            const unsigned nin = sh.nin;
            auto place = [&](auto px) {
                constexpr int PX = decltype(px)::value;
                if ((int)threadIdx.x >= (int)cnt) return;
                unsigned long long kk[PX];
                unsigned char st[PX];
                unsigned r[PX];
#pragma unroll
                for (int u = 0; u < PX; ++u) {
                    const int i = threadIdx.x + u * NT;
                    st[u] = i < (int)cnt ? needf[i] : 2;
                    kk[u] = i < (int)cnt ? cand[i] : 0ull;
                    r[u] = 0;
                }
                for (int j = 0; j < (int)cnt; ++j) {
                    const unsigned char sj = needf[j];
                    const unsigned long long kj = cand[j];
#pragma unroll
                    for (int u = 0; u < PX; ++u) r[u] += (sj == st[u] && kj < kk[u]) ? 1u : 0u;
                }
#pragma unroll
                for (int u = 0; u < PX; ++u) {
                    if (st[u] == 2) continue;
                    const unsigned pos = st[u] == 0 ? r[u] : nin + r[u];
                    if (pos < (unsigned)PP)
                        probes[(int64_t)q * P + pos] = (int32_t)(kk[u] & 0xffffffffu);
                }
            };
            if (cnt <= (unsigned)NT) place(std::integral_constant<int, 1>{});
            else place(std::integral_constant<int, PER>{});
            return;
        }
        if (cnt <= (unsigned)NT) {
            // output position = rank among the candidates (cnt >= PP)
            if (threadIdx.x < cnt) {
                const unsigned long long kk = cand[threadIdx.x];
                unsigned r = 0;
                for (int j = 0; j < (int)cnt; ++j) r += cand[j] < kk ? 1u : 0u;
                if (r < (unsigned)PP) {
                    int32_t id = (int32_t)(kk & 0xffffffffu);
                    if (nan_is_none && (uint32_t)(kk >> 32) == 0xffffffffu) id = -1;
                    probes[(int64_t)q * P + r] = id;
                }
            }
            return;
        }
        int n2 = 1;
        while (n2 < (int)cnt) n2 <<= 1;
        for (int i = (int)cnt + threadIdx.x; i < n2; i += NT) cand[i] = ~0ull;
        __syncthreads();
        bitonic_sort_u64<NT>(cand, n2);
        for (int j = threadIdx.x; j < PP; j += NT) {
            const unsigned long long kk = cand[j];
            int32_t id = (int32_t)(kk & 0xffffffffu);
            if (nan_is_none && (uint32_t)(kk >> 32) == 0xffffffffu) id = -1;
            probes[(int64_t)q * P + j] = id;
        }
        return;
    }

    // --- fallback: exact scores, selection by (score, id).  With T known (more
    // candidates than the candidate array holds) only the candidates are scored:
    // every other centroid's exact score is above T, and at least P centroids
    // (those with an upper bound <= T) score <= T, so +inf in their place changes
    // nothing among the P smallest.
    __syncthreads();
    for (int c = threadIdx.x; c < L; c += NT) {
        bool need = true;
        if (have_t) {
            float lo, hi;
            bounds(c, &lo, &hi);
            need = (lo != lo ? 0u : float_key(lo)) <= t_all;
        }
        srow[c] = need ? exact_score(qs, C + (int64_t)c * ldc, D, metric, nrm)
                       : __int_as_float(0x7f800000);
    }
    __syncthreads();
    const uint32_t kth =
        block_radix_select([&](int c) { return float_key(srow[c]); }, L, (unsigned)PP, sh);
    if (threadIdx.x == 0) {
        sh.count = 0;
        sh.count2 = 0;
    }
    __syncthreads();
    for (int c = threadIdx.x; c < L; c += NT)
        if (float_key(srow[c]) < kth) atomicAdd(&sh.count, 1u);
    __syncthreads();
    const unsigned m_less = sh.count;
    const unsigned tie_need = (unsigned)PP - m_less;
    // ordered compaction: keys < kth, then the first tie_need ids with key == kth
    const bool sorted = PP <= SEL_SORT_MAX;
    unsigned out_pos = 0, ties_taken = 0;
    for (int c0 = 0; c0 < L; c0 += NT) {
        const int c = c0 + threadIdx.x;
        const uint32_t k = c < L ? float_key(srow[c]) : 0xffffffffu;
        const bool tie = c < L && k == kth;
        unsigned tie_tot;
        const unsigned tie_off = block_flag_scan(tie, &tie_tot, sh);
        const bool take = c < L && (k < kth || (tie && ties_taken + tie_off < tie_need));
        unsigned take_tot;
        const unsigned off = block_flag_scan(take, &take_tot, sh);
        if (take) {
            if (sorted)
                cand[out_pos + off] = ((unsigned long long)k << 32) | (unsigned)c;
            else
                probes[(int64_t)q * P + out_pos + off] = c;
        }
        out_pos += take_tot;
        ties_taken += tie_tot;
    }
    __syncthreads();
    if (sorted) {
        int n2 = 1;
        while (n2 < PP) n2 <<= 1;
        for (int i = PP + threadIdx.x; i < n2; i += NT) cand[i] = ~0ull;
        __syncthreads();
        bitonic_sort_u64<NT>(cand, n2);
        for (int j = threadIdx.x; j < PP; j += NT) {
            const unsigned long long kk = cand[j];
            int32_t id = (int32_t)(kk & 0xffffffffu);
            if (nan_is_none && (uint32_t)(kk >> 32) == 0xffffffffu) id = -1;
            probes[(int64_t)q * P + j] = id;
        }
    }
}

namespace {
template <int NT, int CAP>
size_t select_smem_bytes_t(int L, int D) {
    return sizeof(float) * (size_t)((D + 3) & ~3) + sizeof(unsigned long long) * CAP +
           sizeof(float2) * CAP + CAP + sizeof(uint32_t) * sel_area_words<NT, CAP>(L);
}
}  // namespace

size_t select_smem_bytes(int L, int D) {
    return std::max(select_smem_bytes_t<SEL_SMALL_NT, SEL_SMALL_CAP>(L, D),
                    select_smem_bytes_t<SEL_LARGE_NT, SEL_LARGE_CAP>(L, D));
}

int select_max_dim() { return 8192; }

namespace {
constexpr int PS_BLOCK = 256;

// Exact unified scores of given (query, centroid) pairs, one block per query:
// the pairs of a query are spread over the warps, ceil(n / 8) per warp, each
// scored by warp_exact_scores (the reference's arithmetic and summation order).
// probes[q * P + j] < 0 or >= L scores +inf.
__global__ void __launch_bounds__(PS_BLOCK) probe_scores_kernel(
    const float* __restrict__ Q, int64_t ldq, const float* __restrict__ C, int64_t ldc, int L,
    const int32_t* __restrict__ probes, int P, int D, int metric, int normalized,
    float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char ps_smem[];
    float* qs = reinterpret_cast<float*>(ps_smem);                       // round_up(D, 4) floats
    float* stage_all = qs + ((D + 3) & ~3);                               // 8 tiles
    const int q = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* qrow = Q + (int64_t)q * ldq;
    for (int i = threadIdx.x; i < D; i += PS_BLOCK) qs[i] = qrow[i];
    __syncthreads();
    const bool nrm = normalized != 0;
    float* stage = stage_all + warp * kExactTileFloats;
    const int32_t* pr = probes + (int64_t)q * P;
    float* o = out + (int64_t)q * P;
    for (int r0 = 0; r0 < P; r0 += PS_BLOCK) {
        const int n = P - r0 < PS_BLOCK ? P - r0 : PS_BLOCK;
        const int G = (n + PS_BLOCK / 32 - 1) / (PS_BLOCK / 32);
        if (warp * G >= n) continue;  // warp-uniform
        const int i = warp * G + lane;
        const bool mine = lane < G && i < n;
        int c = mine ? pr[r0 + i] : -1;
        if (c >= L) c = -1;
        float r;
        if (G <= 8) r = warp_exact_scores<4>(qs, C, ldc, D, metric, nrm, c, stage, lane);
        else if (G <= 16) r = warp_exact_scores<2>(qs, C, ldc, D, metric, nrm, c, stage, lane);
        else r = warp_exact_scores<1>(qs, C, ldc, D, metric, nrm, c, stage, lane);
        if (mine) o[r0 + i] = c >= 0 ? r : __int_as_float(0x7f800000);
    }
}
}  // namespace

cudaError_t launch_probe_scores(const float* Q, int64_t ldq, const float* C, int64_t ldc, int L,
                                const int32_t* probes, int64_t nq, int P, int D, int metric,
                                int normalized, float* out, cudaStream_t st) {
    if (nq <= 0 || P <= 0) return cudaSuccess;
    const size_t smem = sizeof(float) * ((size_t)((D + 3) & ~3) +
                                         (size_t)(PS_BLOCK / 32) * kExactTileFloats);
    cudaError_t e = cudaFuncSetAttribute(probe_scores_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    probe_scores_kernel<<<(unsigned)nq, PS_BLOCK, smem, st>>>(Q, ldq, C, ldc, L, probes, P, D,
                                                              metric, normalized, out);
    return cudaGetLastError();
}

cudaError_t launch_select_probes(float* S, int64_t lds, const float* Q, int64_t ldq, const float* C,
                                 int64_t ldc, const float* qn, const float* qn2, const float* cn,
                                 const float* cn2, int nq, int L, int D, int metric,
                                 int normalized, float beta, float gamma, int P, int flags,
                                 int32_t* probes, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    auto run = [&](auto kernel, int nt, size_t smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        kernel<<<nq, nt, smem, st>>>(S, lds, Q, ldq, C, ldc, qn, qn2, cn, cn2, L, D, metric,
                                     normalized, beta, gamma, P, flags, probes);
        return cudaGetLastError();
    };
    if ((P < L ? P : L) <= SEL_SMALL_P)
        return run(select_probes_kernel<SEL_SMALL_NT, SEL_SMALL_CAP, SEL_SMALL_MINB>, SEL_SMALL_NT,
                   select_smem_bytes_t<SEL_SMALL_NT, SEL_SMALL_CAP>(L, D));
    return run(select_probes_kernel<SEL_LARGE_NT, SEL_LARGE_CAP, 3>, SEL_LARGE_NT,
               select_smem_bytes_t<SEL_LARGE_NT, SEL_LARGE_CAP>(L, D));
}

}  // namespace m3g
