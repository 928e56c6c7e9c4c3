// kernels_kmeans.h -- launchers of k_kmeans.cu (internal to libm3gpu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace m3g {

// Rows per chunk of the stable counting sort for n rows and L clusters.
int64_t sort_chunk_rows(int64_t n, int L);
// perm[start[l] .. start[l+1]) = rows assigned to l, ascending.  counts holds
// ceil(n/chunk) * L ints, totals L ints, start L+1 int64s, perm n int64s.
cudaError_t launch_stable_cluster_sort(const int32_t* assign, int64_t n, int L, int64_t chunk,
                                       int32_t* counts, int32_t* totals, int64_t* start,
                                       int64_t* perm, cudaStream_t st);
cudaError_t launch_centroid_update(const float* X, int64_t ldx, const int64_t* perm,
                                   const int64_t* start, int L, int d, float* C, int64_t ldc,
                                   cudaStream_t st);

cudaError_t launch_gather_rows(const float* src, int64_t lds, const int64_t* idx, int64_t n,
                               int width, float* dst, int64_t ldd, cudaStream_t st);
cudaError_t launch_scatter_rows(const float* src, int64_t lds, const int64_t* dst_rows, int64_t n,
                                int width, float* dst, int64_t ldd, cudaStream_t st);
// Segmented 2-means of the split pass: per row its segment's exact nearest of
// two centroids (side 0 / 1, -1 if both scores are NaN); per (segment, side,
// dim) the fp64 mean over the segment's rows on that side, in row order.
cudaError_t launch_seg2_assign(const float* X, int64_t ld, const int32_t* row_seg, int64_t n,
                               const float* C2, int dim, int metric, int normalized,
                               int32_t* side, cudaStream_t st);
cudaError_t launch_seg2_update(const float* X, int64_t ld, const int64_t* seg_off, int nseg,
                               const int32_t* side, int dim, float* C2, cudaStream_t st);
// Moves arena rows src[i] -> dst[i] (disjoint sets): row words, norm, id and
// tombstone.
cudaError_t launch_move_rows(float* vecs, int64_t words, float* nrm, int64_t* ids, uint8_t* alive,
                             const int64_t* src, const int64_t* dst, int64_t n, cudaStream_t st);
// bf16 rows of the list arena: values rounded to bf16 in place (kept as fp32),
// packed fp32 -> bf16 rows (columns dim .. ldd zero), and widened back.
cudaError_t launch_round_bf16_rows(float* X, int64_t ld, int64_t n, int dim, cudaStream_t st);
cudaError_t launch_pack_bf16_rows(const float* src, int64_t lds, int64_t n, int dim,
                                  __nv_bfloat16* dst, int64_t ldd, cudaStream_t st);
cudaError_t launch_unpack_bf16_rows(const __nv_bfloat16* src, int64_t lds, int64_t n, int dim,
                                    float* dst, int64_t ldd, cudaStream_t st);
cudaError_t launch_gather_i64(const int64_t* src, const int64_t* idx, int64_t n, int64_t* dst,
                              cudaStream_t st);
cudaError_t launch_gather_f32(const float* src, const int64_t* idx, int64_t n, float* dst,
                              cudaStream_t st);
cudaError_t launch_gather_u8(const uint8_t* src, const int64_t* idx, int64_t n, uint8_t* dst,
                             cudaStream_t st);
cudaError_t launch_scatter_i64(const int64_t* src, const int64_t* idx, int64_t n, int64_t* dst,
                               cudaStream_t st);
cudaError_t launch_set_bytes(uint8_t* dst, const int64_t* idx, int64_t n, uint8_t v,
                             cudaStream_t st);
cudaError_t launch_iota_rows(int32_t* out, int64_t nrows, int width, cudaStream_t st);
cudaError_t launch_broadcast_row(const int32_t* row, int width, int64_t nrows, int32_t* out,
                                 cudaStream_t st);
cudaError_t launch_probed_rows(const int32_t* lcount, const int32_t* list_len, int L, int gmax,
                               unsigned long long* out_rows, unsigned long long* out_pairs,
                               unsigned long long* out_streamed, cudaStream_t st);

}  // namespace m3g
