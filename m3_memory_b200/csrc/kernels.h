// kernels.h -- host-side launchers of the m3gpu CUDA kernels (internal to
// libm3gpu; the public C ABI is include/m3gpu.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace m3g {

// ---- coarse quantizer (k_coarse.cu) ----
void launch_row_norms(const float* X, int64_t ld, int64_t n, int d, float* nrm_up, float* nrm2,
                      cudaStream_t st);
void launch_sgemm_nt(const float* A, int64_t lda, const float* B, int64_t ldb, float* S,
                     int64_t lds, int M, int N, int K, cudaStream_t st);
float sgemm_error_beta(int K);
// The GEMV form of launch_sgemm_nt for M <= 8 rows of A (the same error bound);
// gemv_fits tells whether it takes the operands (K and B's rows in 16-byte units).
bool gemv_fits(const float* A, int64_t lda, const float* B, int64_t ldb, int M, int K);
void launch_gemv_nt(const float* A, int64_t lda, const float* B, int64_t ldb, float* S,
                    int64_t lds, int M, int N, int K, int num_sms, cudaStream_t st);
size_t select_smem_bytes(int L, int D);
int select_max_dim();
// flags of launch_select_probes
constexpr int kSelectNanIsNone = 1;  // P == 1: -1 where every score is NaN
constexpr int kSelectSetOnly = 2;    // each row holds the top-P set in no particular order
cudaError_t launch_select_probes(float* S, int64_t lds, const float* Q, int64_t ldq, const float* C,
                                 int64_t ldc, const float* qn, const float* qn2, const float* cn,
                                 const float* cn2, int nq, int L, int D, int metric,
                                 int normalized, float beta, float gamma, int P, int flags,
                                 int32_t* probes, cudaStream_t st);

// ---- coarse GEMM on the tensor cores (k_gemm_tc.cu) ----
int gemm_tc_kdim(int dpad);            // K' of the split operands (3 dpad, padded to 64)
float gemm_tc_error_beta(int dpad);    // |approx dot - exact| <= beta * ||a|| ||b||
int gemm_tc_box_rows_a();
int gemm_tc_box_rows_b();
int gemm_tc_box_k();
cudaError_t launch_split3(const float* X, int64_t ld, int64_t n, int dpad, int kp,
                          __nv_bfloat16* out, bool centroid_side, cudaStream_t st);
// Row norms of n query rows (as launch_row_norms) and, with q3, their query-side
// split operand rows (as launch_split3), from one read of each row.
cudaError_t launch_query_prep(const float* X, int64_t ld, int64_t n, int d, int dpad, int kp,
                              __nv_bfloat16* q3, float* nrm_up, float* nrm2, cudaStream_t st);
cudaError_t launch_gemm_tc(const CUtensorMap& mapA, const CUtensorMap& mapB, float* S, int64_t lds,
                           int M, int N, int kp, int* err, cudaStream_t st);

// 2-D tiled tensor map (host; driver entry point fetched through the runtime).
void encode_tma_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                   uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                   CUtensorMapSwizzle swizzle);

// ---- list scan (k_scan.cu) ----
struct ScanItem {
    int32_t list;        // cluster id
    int32_t pair_begin;  // first (query, probe slot) pair of this item in the pair arrays
    int32_t npairs;      // number of queries in the item (<= gmax)
    int32_t row_begin;   // first row of the list the item scans
    int32_t nrows;       // rows it scans; -1: to the end of the list
    // Row tiles of a long list (tile_nt > 0): the item is tile tile_t of tile_nt,
    // its pair i writes its partial top-k to tile partial tile_out + i tile_nt +
    // tile_t (an index into the tile region of the partial lists, which starts at
    // ScanArgs::tile_base), and the last tile to finish merges the pair's
    // tile_nt lists into its own (query, probe slot) partial list.
    int32_t tile_out;
    int32_t tile_t;
    int32_t tile_nt;
};

// Row boxes of the list arena for the scans: 2-D tensor maps over the arena
// viewed as [rows, dpad] fp32, box width 32 floats (128 B, SWIZZLE_128B) and
// heights 128 / 64 / 32 / 16 / 8 rows.
struct RowMaps {
    CUtensorMap m128, m64, m32, m16, m8;
};

struct ScanArgs {
    const float* Q;          // [nq, dpad] queries (rows padded with zeros)
    int dpad;                // floats per arena / query row (multiple of 4)
    const int64_t* list_off; // [L] first arena row of each list
    const int32_t* list_len; // [L] rows in each list
    const uint8_t* alive;    // [arena rows] tombstones (0 = erased)
    const float* rnorm2;     // [arena rows] ||x||^2 (non-normalised COSINE only)
    const float* qnorm2;     // [nq] ||q||^2 (non-normalised COSINE only)
    const ScanItem* items;
    const int32_t* n_items;  // device count
    int32_t* item_counter;   // device, zeroed before launch
    uint32_t* qbound;        // [nq] ~(score key) bounding each query's k-th best score, zeroed
                             // (no bound) before launch; null: not used
    const int32_t* pair_q;
    const int32_t* pair_slot;
    int k, P, metric, normalized;
    float* part_score;       // [nq, P, k]
    int64_t* part_row;       // [nq, P, k] arena row, -1 for empty
    int* err;
    // test hook (tensor-core scan): when nonzero, the scheduler first waits this
    // long on a barrier nothing arrives at, records the timeout and ends the scan
    uint64_t test_wait_ns;
    // row tiles (tensor-core scan): partial index of the tile region and, per
    // tiled pair, a counter of its finished tiles (zeroed before launch)
    int64_t tile_base;
    int32_t* tile_cnt;
};

int scan_kmax();
int scan_gmax_for_dim(int dpad);
cudaError_t launch_list_scan(const RowMaps& maps, const ScanArgs& a, int gmax, int grid,
                             cudaStream_t st);

// The tensor-core scan (k_scan_tc.cu): every metric, k <= 128, items of up to
// scan_tc_gmax(k) queries; rows fp32 or (bf16_rows) bf16.  Squared L2 comes out
// as a ranking estimate that the merge must rescore (MergeRescore).
bool scan_tc_supported(int metric, int k);
int scan_tc_gmax(int k);
cudaError_t launch_list_scan_tc(const RowMaps& maps, const ScanArgs& a, bool bf16_rows, int grid,
                                cudaStream_t st);

// Work list: per-list counts of (query, probe) pairs, items, and the pairs
// grouped by list.  list_order lists the clusters longest first.  With
// skip_len ([L] rows per list), pairs probing an empty list are left out (their
// partial lists must then be cleared beforehand).  With tile_rows > 0 (a
// multiple of 128; the tensor-core scan only) a list longer than tile_rows and
// probed by at most two query groups is scanned in row tiles of tile_rows, each
// group once per tile, as long as its tile partial lists fit the tile region of
// tile_cap lists (longest lists first); list_len gives the rows per list.
// plan: scratch of 6 L int32.
cudaError_t launch_build_worklist(const int32_t* probes, int nq, int P, int L,
                                  const int32_t* list_order, int gmax, int32_t* lcount,
                                  int32_t* lstart, int32_t* lcursor, ScanItem* items,
                                  int32_t* n_items, int32_t* pair_q, int32_t* pair_slot,
                                  int32_t* plan, cudaStream_t st, const int32_t* skip_len = nullptr,
                                  const int32_t* list_len = nullptr, int tile_rows = 0,
                                  int tile_cap = 0);

// Exact squared-L2 rescoring of a merge's winners: the reference's sum of
// (q_i - x_i)^2 in index order (AgentMemory/M3/src/base.cpp:12-20) over the
// arena rows (fp32, or bf16 widened to fp32) and the queries.
struct MergeRescore {
    const float* Q;        // [nq, ldq] queries
    int64_t ldq;
    const void* rows;      // arena rows, row_ld elements apart
    int64_t row_ld;
    int dim;
    int bf16_rows;
};

// Final merge of the per-(query, probe) partial top-k into the answer; with rs,
// the winners' scores are replaced by exact squared-L2 scores and re-sorted.
cudaError_t launch_merge_topk(const float* part_score, const int64_t* part_row,
                              const int64_t* row_ids, int nq, int P, int k, int64_t* out_ids,
                              float* out_scores, int32_t* out_counts, cudaStream_t st,
                              const MergeRescore* rs = nullptr);

// Merge of per-shard answers [nshard, nq, k] (scores ascending per row, ids,
// -1 / +inf padding) into [nq, k]; ties broken by (shard, position).
// Empty partial top-k lists (+inf, -1): for probe slots a search skips.
cudaError_t launch_clear_partials(float* part_score, int64_t* part_row, int64_t n, cudaStream_t st);

// Exact unified scores (the reference's arithmetic) of the pairs (q, probes[q, j]),
// +inf where the probe is out of [0, L).
cudaError_t launch_probe_scores(const float* Q, int64_t ldq, const float* C, int64_t ldc, int L,
                                const int32_t* probes, int64_t nq, int P, int D, int metric,
                                int normalized, float* out, cudaStream_t st);

// The same over one gathered buffer: shard s's record starts at packed + s *
// shard_bytes and holds its [nq, k] fp32 scores, then at ids_offset its [nq, k]
// int64 ids (both multiples of 8 bytes).
cudaError_t launch_merge_shards_packed(const unsigned char* packed, int nshard, int nq, int k,
                                       int64_t shard_bytes, int64_t ids_offset, int64_t* out_ids,
                                       float* out_scores, int32_t* out_counts, cudaStream_t st);
cudaError_t launch_merge_shards(const float* scores, const int64_t* ids, int nshard, int nq, int k,
                                int64_t* out_ids, float* out_scores, int32_t* out_counts,
                                cudaStream_t st);

}  // namespace m3g
