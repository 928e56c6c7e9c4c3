// k_kmeans.cu -- k-means M-step and the row-movement kernels of the list arena.
//
// The reference has no k-means (AgentMemory/M3/src/m3_index.cpp:304-311 is a
// TODO; centroids always come from the caller).  The update rule specified here:
// each centroid becomes the fp64 sum of its rows, taken in ascending row order,
// divided by the count in fp64 and rounded to fp32; an empty cluster keeps its
// previous centroid.  The running-mean form of the same idea is in the
// reference's MultiLevelIndex::insert (AgentMemory/M3/src/m3_multi_level.cpp:131-148).
//
// The fixed summation order makes the result bit-reproducible: rows are first
// put in (cluster, row) order by a stable counting sort, then one thread per
// (cluster, dim) sums its cluster's rows sequentially -- a segmented reduction
// with no atomics on the data path.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "score.cuh"
#include "kernels_kmeans.h"

namespace m3g {
namespace {

__global__ void chunk_hist_kernel(const int32_t* __restrict__ assign, int64_t n, int L,
                                  int64_t chunk, int32_t* __restrict__ counts,
                                  int32_t* __restrict__ totals) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = assign[i];
        if (l < 0 || l >= L) continue;
        atomicAdd(&counts[(i / chunk) * L + l], 1);
        atomicAdd(&totals[l], 1);
    }
}

constexpr int SCAN_THREADS = 1024;

// Exclusive scan of totals[0..L) into start[0..L]; one block.
__global__ void __launch_bounds__(SCAN_THREADS) exclusive_scan_kernel(
    const int32_t* __restrict__ totals, int L, int64_t* __restrict__ start) {
    __shared__ int64_t sp[SCAN_THREADS];
    const int t = threadIdx.x;
    const int per = (L + SCAN_THREADS - 1) / SCAN_THREADS;
    const int b = t * per, e = min(L, b + per);
    int64_t s = 0;
    for (int i = b; i < e; ++i) s += totals[i];
    sp[t] = s;
    __syncthreads();
    for (int o = 1; o < SCAN_THREADS; o <<= 1) {
        const int64_t v = t >= o ? sp[t - o] : 0;
        __syncthreads();
        sp[t] += v;
        __syncthreads();
    }
    int64_t base = sp[t] - s;
    for (int i = b; i < e; ++i) {
        start[i] = base;
        base += totals[i];
    }
    if (t == SCAN_THREADS - 1) start[L] = sp[t];
}

// counts[c][l] := first output position of cluster l's rows from chunk c.
__global__ void chunk_offsets_kernel(int32_t* __restrict__ counts, int64_t nchunks, int L,
                                     const int64_t* __restrict__ start) {
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= L) return;
    int64_t run = start[l];
    for (int64_t c = 0; c < nchunks; ++c) {
        const int32_t v = counts[c * L + l];
        counts[c * L + l] = (int32_t)run;
        run += v;
    }
}

// One warp per chunk, rows in ascending order: stable placement.
__global__ void chunk_scatter_kernel(const int32_t* __restrict__ assign, int64_t n, int L,
                                     int64_t chunk, int64_t nchunks, int32_t* __restrict__ cursor,
                                     int64_t* __restrict__ perm) {
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (c >= nchunks) return;
    const int64_t b = c * chunk, e = min(n, b + chunk);
    const unsigned lt = (1u << lane) - 1u;
    int32_t* cur = cursor + c * L;
    for (int64_t base = b; base < e; base += 32) {
        const int64_t r = base + lane;
        int l = r < e ? assign[r] : -1;
        if (l >= L) l = -1;
        const unsigned peers = __match_any_sync(0xffffffffu, l);
        const int rank = __popc(peers & lt);
        const int leader = __ffs(peers) - 1;
        int32_t pos0 = 0;
        if (l >= 0) pos0 = cur[l];
        __syncwarp();
        if (l >= 0) {
            perm[pos0 + rank] = r;
            if (lane == leader) cur[l] = pos0 + __popc(peers);
        }
        __syncwarp();
    }
}

// C[l][d] = fp32(fp64 sum over the cluster's rows, ascending, / count).
__global__ void centroid_update_kernel(const float* __restrict__ X, int64_t ldx,
                                       const int64_t* __restrict__ perm,
                                       const int64_t* __restrict__ start, int d,
                                       float* __restrict__ C, int64_t ldc) {
    const int l = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    const int64_t b = start[l], e = start[l + 1];
    if (b == e) return;
    double acc = 0.0;
    for (int64_t i = b; i < e; ++i) acc = acc + (double)X[perm[i] * ldx + j];
    C[(int64_t)l * ldc + j] = (float)(acc / (double)(e - b));
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t lds,
                                   const int64_t* __restrict__ idx, int64_t n, int width,
                                   float* __restrict__ dst, int64_t ldd) {
    const int64_t r = blockIdx.y;
    if (r >= n) return;
    const int64_t s = idx[r];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < width; j += gridDim.x * blockDim.x)
        dst[r * ldd + j] = src[s * lds + j];
}

__global__ void scatter_rows_kernel(const float* __restrict__ src, int64_t lds,
                                    const int64_t* __restrict__ dst_rows, int64_t n, int width,
                                    float* __restrict__ dst, int64_t ldd) {
    const int64_t r = blockIdx.y;
    if (r >= n) return;
    const int64_t t = dst_rows[r];
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < width; j += gridDim.x * blockDim.x)
        dst[t * ldd + j] = src[r * lds + j];
}

template <class T>
__global__ void gather_elems_kernel(const T* __restrict__ src, const int64_t* __restrict__ idx,
                                    int64_t n, T* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[idx[i]];
}

template <class T>
__global__ void scatter_elems_kernel(const T* __restrict__ src, const int64_t* __restrict__ idx,
                                     int64_t n, T* __restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[idx[i]] = src[i];
}

__global__ void set_bytes_kernel(uint8_t* __restrict__ dst, const int64_t* __restrict__ idx,
                                 int64_t n, uint8_t v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[idx[i]] = v;
}

__global__ void iota_rows_kernel(int32_t* __restrict__ out, int64_t nrows, int width) {
    const int64_t n = nrows * width;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int32_t)(i % width);
}

__global__ void broadcast_row_kernel(const int32_t* __restrict__ row, int width, int64_t nrows,
                                     int32_t* __restrict__ out) {
    const int64_t n = nrows * width;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = row[i % width];
}

// Sum of the lengths of the lists a batch probes (for the scan's byte count),
// the pairs, and the rows the scan's items stream (each list once per group of
// up to gmax of its queries).
__global__ void probed_rows_kernel(const int32_t* __restrict__ lcount,
                                   const int32_t* __restrict__ list_len, int L, int gmax,
                                   unsigned long long* __restrict__ out_rows,
                                   unsigned long long* __restrict__ out_pairs,
                                   unsigned long long* __restrict__ out_streamed) {
    unsigned long long rows = 0, pairs = 0, streamed = 0;
    for (int l = blockIdx.x * blockDim.x + threadIdx.x; l < L; l += gridDim.x * blockDim.x) {
        const int c = lcount[l];
        if (c > 0) {
            rows += (unsigned long long)list_len[l];
            streamed += (unsigned long long)list_len[l] * (unsigned long long)((c + gmax - 1) / gmax);
        }
        pairs += (unsigned long long)c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        rows += __shfl_xor_sync(0xffffffffu, rows, o);
        pairs += __shfl_xor_sync(0xffffffffu, pairs, o);
        streamed += __shfl_xor_sync(0xffffffffu, streamed, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(out_rows, rows);
        atomicAdd(out_pairs, pairs);
        atomicAdd(out_streamed, streamed);
    }
}

inline int grid_for(int64_t n, int block) {
    int64_t g = (n + block - 1) / block;
    if (g > 65535) g = 65535;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace

int64_t sort_chunk_rows(int64_t n, int L) {
    int64_t chunk = 4096;
    const int64_t budget = int64_t(1) << 26;  // counts matrix entries
    while ((n + chunk - 1) / chunk * (int64_t)L > budget) chunk *= 2;
    return chunk;
}

cudaError_t launch_stable_cluster_sort(const int32_t* assign, int64_t n, int L, int64_t chunk,
                                       int32_t* counts, int32_t* totals, int64_t* start,
                                       int64_t* perm, cudaStream_t st) {
    const int64_t nchunks = (n + chunk - 1) / chunk;
    cudaError_t e;
    if ((e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * (size_t)(nchunks * L), st))) return e;
    if ((e = cudaMemsetAsync(totals, 0, sizeof(int32_t) * (size_t)L, st))) return e;
    if (n > 0) chunk_hist_kernel<<<grid_for(n, 256), 256, 0, st>>>(assign, n, L, chunk, counts, totals);
    exclusive_scan_kernel<<<1, SCAN_THREADS, 0, st>>>(totals, L, start);
    chunk_offsets_kernel<<<(L + 255) / 256, 256, 0, st>>>(counts, nchunks, L, start);
    if (n > 0)
        chunk_scatter_kernel<<<(unsigned)((nchunks + 7) / 8), 256, 0, st>>>(assign, n, L, chunk,
                                                                           nchunks, counts, perm);
    return cudaGetLastError();
}

cudaError_t launch_centroid_update(const float* X, int64_t ldx, const int64_t* perm,
                                   const int64_t* start, int L, int d, float* C, int64_t ldc,
                                   cudaStream_t st) {
    if (L <= 0) return cudaSuccess;
    dim3 grid((d + 127) / 128, L);
    centroid_update_kernel<<<grid, 128, 0, st>>>(X, ldx, perm, start, d, C, ldc);
    return cudaGetLastError();
}

namespace {
__global__ void round_bf16_rows_kernel(float* __restrict__ X, int64_t ld, int64_t n, int dim) {
    const int64_t total = n * dim;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        float* p = X + (t / dim) * ld + t % dim;
        *p = __bfloat162float(__float2bfloat16_rn(*p));
    }
}

__global__ void pack_bf16_rows_kernel(const float* __restrict__ src, int64_t lds, int64_t n, int dim,
                                      __nv_bfloat16* __restrict__ dst, int64_t ldd) {
    const int64_t total = n * ldd;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ldd, i = t % ldd;
        dst[r * ldd + i] = i < dim ? __float2bfloat16_rn(src[r * lds + i]) : __float2bfloat16_rn(0.f);
    }
}

__global__ void unpack_bf16_rows_kernel(const __nv_bfloat16* __restrict__ src, int64_t lds,
                                        int64_t n, int dim, float* __restrict__ dst, int64_t ldd) {
    const int64_t total = n * ldd;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ldd, i = t % ldd;
        dst[r * ldd + i] = i < dim ? __bfloat162float(src[r * lds + i]) : 0.f;
    }
}

unsigned grid_for(int64_t total) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 8192));
}
}  // namespace

// ---------------------------------------------------------------------------
// Segmented 2-means (the split pass): segment s = rows [seg_off[s],
// seg_off[s+1]) of X, two centroids per segment in C2 [2 nseg, ld].  The same
// rules as the k-means above, per segment: exact nearest_clusters assignment
// (strict '<', centroid 0 wins ties, -1 if both scores are NaN) and fp64 means
// in ascending row order, an empty side keeping its centroid.
// ---------------------------------------------------------------------------
namespace {
__global__ void seg2_assign_kernel(const float* __restrict__ X, int64_t ld,
                                   const int32_t* __restrict__ row_seg, int64_t n,
                                   const float* __restrict__ C2, int dim, int metric,
                                   int normalized, int32_t* __restrict__ side) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    const int s = row_seg[r];
    const float* x = X + r * ld;
    const float s0 = exact_score(x, C2 + (int64_t)(2 * s) * ld, dim, metric, normalized != 0);
    const float s1 = exact_score(x, C2 + (int64_t)(2 * s + 1) * ld, dim, metric, normalized != 0);
    float best = __int_as_float(0x7f800000);
    int bid = -1;
    if (s0 < best) {
        best = s0;
        bid = 0;
    }
    if (s1 < best) bid = 1;
    side[r] = bid;
}

__global__ void seg2_update_kernel(const float* __restrict__ X, int64_t ld,
                                   const int64_t* __restrict__ seg_off, int nseg,
                                   const int32_t* __restrict__ side, int dim,
                                   float* __restrict__ C2) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    const int s = blockIdx.y >> 1, which = blockIdx.y & 1;
    if (d >= dim || s >= nseg) return;
    double acc = 0.0;
    int64_t cnt = 0;
    for (int64_t r = seg_off[s]; r < seg_off[s + 1]; ++r)
        if (side[r] == which) {
            acc += (double)X[r * ld + d];
            ++cnt;
        }
    if (cnt > 0) C2[(int64_t)(2 * s + which) * ld + d] = (float)(acc / (double)cnt);
}
}  // namespace

cudaError_t launch_seg2_assign(const float* X, int64_t ld, const int32_t* row_seg, int64_t n,
                               const float* C2, int dim, int metric, int normalized,
                               int32_t* side, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    seg2_assign_kernel<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(X, ld, row_seg, n, C2, dim,
                                                                    metric, normalized, side);
    return cudaGetLastError();
}

cudaError_t launch_seg2_update(const float* X, int64_t ld, const int64_t* seg_off, int nseg,
                               const int32_t* side, int dim, float* C2, cudaStream_t st) {
    if (nseg <= 0) return cudaSuccess;
    for (int s0 = 0; s0 < nseg; s0 += 32768) {
        const int m = std::min(32768, nseg - s0);
        dim3 grid((unsigned)((dim + 127) / 128), (unsigned)(2 * m));
        seg2_update_kernel<<<grid, 128, 0, st>>>(X, ld, seg_off + s0, m, side, dim,
                                                 C2 + (int64_t)(2 * s0) * ld);
    }
    return cudaGetLastError();
}

namespace {
// Row moves inside one arena (disjoint source and destination rows): the row
// words, the norm, the id and the tombstone of row src[i] go to row dst[i].
__global__ void move_rows_kernel(float* __restrict__ vecs, int64_t words, float* __restrict__ nrm,
                                 int64_t* __restrict__ ids, uint8_t* __restrict__ alive,
                                 const int64_t* __restrict__ src, const int64_t* __restrict__ dst,
                                 int64_t n) {
    const int64_t r = blockIdx.y + (int64_t)blockIdx.z * 65535;
    if (r >= n) return;
    const int64_t s = src[r], t = dst[r];
    for (int64_t j = blockIdx.x * blockDim.x + threadIdx.x; j < words; j += gridDim.x * blockDim.x)
        vecs[t * words + j] = vecs[s * words + j];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        nrm[t] = nrm[s];
        ids[t] = ids[s];
        alive[t] = alive[s];
    }
}
}  // namespace

cudaError_t launch_move_rows(float* vecs, int64_t words, float* nrm, int64_t* ids, uint8_t* alive,
                             const int64_t* src, const int64_t* dst, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int64_t z = (n + 65534) / 65535;
    if (z > 65535) return cudaErrorInvalidValue;
    dim3 grid((unsigned)std::min<int64_t>((words + 255) / 256, 8), (unsigned)std::min<int64_t>(n, 65535),
              (unsigned)z);
    move_rows_kernel<<<grid, 256, 0, st>>>(vecs, words, nrm, ids, alive, src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_round_bf16_rows(float* X, int64_t ld, int64_t n, int dim, cudaStream_t st) {
    if (n <= 0 || dim <= 0) return cudaSuccess;
    round_bf16_rows_kernel<<<grid_for(n * dim), 256, 0, st>>>(X, ld, n, dim);
    return cudaGetLastError();
}

cudaError_t launch_pack_bf16_rows(const float* src, int64_t lds, int64_t n, int dim,
                                  __nv_bfloat16* dst, int64_t ldd, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    pack_bf16_rows_kernel<<<grid_for(n * ldd), 256, 0, st>>>(src, lds, n, dim, dst, ldd);
    return cudaGetLastError();
}

cudaError_t launch_unpack_bf16_rows(const __nv_bfloat16* src, int64_t lds, int64_t n, int dim,
                                    float* dst, int64_t ldd, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    unpack_bf16_rows_kernel<<<grid_for(n * ldd), 256, 0, st>>>(src, lds, n, dim, dst, ldd);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* src, int64_t lds, const int64_t* idx, int64_t n,
                               int width, float* dst, int64_t ldd, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    for (int64_t b = 0; b < n; b += 65535) {
        const int64_t m = std::min<int64_t>(65535, n - b);
        dim3 grid((width + 255) / 256, (unsigned)m);
        gather_rows_kernel<<<grid, 256, 0, st>>>(src, lds, idx + b, m, width, dst + b * ldd, ldd);
    }
    return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const float* src, int64_t lds, const int64_t* dst_rows, int64_t n,
                                int width, float* dst, int64_t ldd, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    for (int64_t b = 0; b < n; b += 65535) {
        const int64_t m = std::min<int64_t>(65535, n - b);
        dim3 grid((width + 255) / 256, (unsigned)m);
        scatter_rows_kernel<<<grid, 256, 0, st>>>(src + b * lds, lds, dst_rows + b, m, width, dst,
                                                  ldd);
    }
    return cudaGetLastError();
}

cudaError_t launch_gather_i64(const int64_t* src, const int64_t* idx, int64_t n, int64_t* dst,
                              cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    gather_elems_kernel<int64_t><<<grid_for(n, 256), 256, 0, st>>>(src, idx, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_gather_f32(const float* src, const int64_t* idx, int64_t n, float* dst,
                              cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    gather_elems_kernel<float><<<grid_for(n, 256), 256, 0, st>>>(src, idx, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_gather_u8(const uint8_t* src, const int64_t* idx, int64_t n, uint8_t* dst,
                             cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    gather_elems_kernel<uint8_t><<<grid_for(n, 256), 256, 0, st>>>(src, idx, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_scatter_i64(const int64_t* src, const int64_t* idx, int64_t n, int64_t* dst,
                               cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    scatter_elems_kernel<int64_t><<<grid_for(n, 256), 256, 0, st>>>(src, idx, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_set_bytes(uint8_t* dst, const int64_t* idx, int64_t n, uint8_t v,
                             cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    set_bytes_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, idx, n, v);
    return cudaGetLastError();
}

cudaError_t launch_iota_rows(int32_t* out, int64_t nrows, int width, cudaStream_t st) {
    if (nrows <= 0 || width <= 0) return cudaSuccess;
    iota_rows_kernel<<<grid_for(nrows * width, 256), 256, 0, st>>>(out, nrows, width);
    return cudaGetLastError();
}

cudaError_t launch_broadcast_row(const int32_t* row, int width, int64_t nrows, int32_t* out,
                                 cudaStream_t st) {
    if (nrows <= 0 || width <= 0) return cudaSuccess;
    broadcast_row_kernel<<<grid_for(nrows * width, 256), 256, 0, st>>>(row, width, nrows, out);
    return cudaGetLastError();
}

cudaError_t launch_probed_rows(const int32_t* lcount, const int32_t* list_len, int L, int gmax,
                               unsigned long long* out_rows, unsigned long long* out_pairs,
                               unsigned long long* out_streamed, cudaStream_t st) {
    probed_rows_kernel<<<grid_for(L, 256), 256, 0, st>>>(lcount, list_len, L, gmax, out_rows,
                                                         out_pairs, out_streamed);
    return cudaGetLastError();
}

}  // namespace m3g
