/* m3gpu.h -- C ABI of libm3gpu, the B200 (sm_100a) engine for the M3 IVF index
 * hot path of AgentMemory's `m3` backend (Leo9660/M3_memory).
 *
 * Each entry point replaces one method of the reference's m3::AsyncEngine
 * (AgentMemory/M3/include/m3_async.h:63-169, bound to Python by
 * AgentMemory/M3/src/bindings_async.cpp:153-588); the citation beside each
 * declaration names the reference interface it stands for.  Only plain
 * pointers, sizes and ints cross this boundary.
 *
 * Conventions
 *   - Every function returns an m3g_status (0 = ok).  On failure the calling
 *     thread's m3g_last_error() holds a message.  The status codes map onto the
 *     reference's C++ exception types: M3G_EINVAL = std::invalid_argument,
 *     M3G_ERANGE = std::out_of_range, M3G_ERUNTIME = std::runtime_error.
 *   - Host pointers are plain host memory (pinned or pageable); functions named
 *     *_device take device pointers of the engine's CUDA device.
 *   - Vectors are row-major float32 [n, dim]; ids are int64.
 *   - Search results are written padded: out_ids[nq*k] / out_scores[nq*k] with
 *     -1 / +inf in unused slots, out_counts[nq] = valid results per query
 *     (the reference returns ragged lists after dropping -1 slots,
 *     AgentMemory/M3/src/m3_index.cpp:444-475).
 *   - Scores are the reference's unified "smaller is better" score
 *     (AgentMemory/M3/include/base.h:22-31): squared L2, -dot, 1-dot, or
 *     1-cosine.
 */
#ifndef M3GPU_H
#define M3GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct m3g_engine m3g_engine;

typedef enum {
    M3G_OK = 0,
    M3G_EINVAL = 1,       /* std::invalid_argument */
    M3G_ERANGE = 2,       /* std::out_of_range */
    M3G_ERUNTIME = 3,     /* std::runtime_error */
    M3G_ECUDA = 4,        /* a CUDA runtime / driver call failed */
    M3G_ENCCL = 5,        /* a collective failed */
    M3G_ETIMEOUT = 6,     /* a bounded device wait ran out */
    M3G_EUNSUPPORTED = 7  /* valid request outside this engine's limits */
} m3g_status;

/* m3::Metric, AgentMemory/M3/include/base.h:10 */
typedef enum { M3G_L2 = 0, M3G_IP = 1, M3G_COSINE = 2 } m3g_metric;

/* Element types of vectors crossing the ABI (m3g_load_cluster) and of an
 * index's list storage (m3g_create_ivf_ex).  The reference stores fp32 only
 * (Cluster::mat_, AgentMemory/M3/include/cluster.h:83). */
typedef enum { M3G_F32 = 0, M3G_BF16 = 1 } m3g_dtype;
#define M3G_STORE_FP32 M3G_F32
#define M3G_STORE_BF16 M3G_BF16

/* Message of the last failing call on this thread ("" if none). */
const char* m3g_last_error(void);
/* ABI version (major * 10000 + minor * 100 + patch). */
int m3g_version(void);

/* AsyncEngine::AsyncEngine / ~AsyncEngine (AgentMemory/M3/src/m3_async.cpp:14-32).
 * The engine binds to the CUDA device current on the calling thread. */
int m3g_engine_create(m3g_engine** out);
int m3g_engine_destroy(m3g_engine* e);
/* Rebind to CUDA device `device` (before any index is created). */
int m3g_set_device(m3g_engine* e, int device);

/* AsyncEngine::start / stop (m3_async.cpp:53-105). */
int m3g_start(m3g_engine* e, int writer_threads, int maintenance_threads);
int m3g_stop(m3g_engine* e);

/* AsyncEngine::set_*_policy (m3_async.cpp:109-119; AsyncQueuePolicy,
 * AsyncSearchPolicy, AsyncMaintenancePolicy at m3_async.h:44-59).  auto_split
 * has no counterpart: when nonzero the maintenance pass also splits lists
 * larger than split_threshold rows (the reference leaves this as a TODO,
 * m3_index.cpp:304-311); 0 keeps the reference's behaviour. */
int m3g_set_queue_policy(m3g_engine* e, size_t capacity, size_t pop_batch_max,
                         int block_on_full);
int m3g_set_search_policy(m3g_engine* e, int default_nprobe, int parallel_queries);
int m3g_set_maintenance_policy(m3g_engine* e, double period_sec, size_t split_threshold,
                               double compact_ratio, int auto_split);

/* The split rule of the maintenance pass (no reference counterpart: its
 * split is a TODO, m3_index.cpp:304-311).  mean_factor > 0: with auto_split on,
 * every pass splits the lists holding more than mean_factor x the mean live
 * rows over all lists (m3g_split_oversized) instead of using split_threshold;
 * niter: 2-means rounds per split (default 5).  m3g_set_maintenance_policy
 * leaves this rule as it is. */
int m3g_set_split_policy(m3g_engine* e, double mean_factor, int niter);

/* AsyncEngine::create_ivf (m3_async.cpp:36-49 -> IVFIndex::set_centroids,
 * m3_index.cpp:98-131).  centroids: [nlist, dim]; nlist may be 0.  Replaces
 * an existing index of the same id. */
int m3g_create_ivf(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                   const float* centroids, int64_t nlist);

/* AsyncEngine::create_ivf with the list storage chosen: M3G_F32 (as
 * m3g_create_ivf) or M3G_BF16, rows kept as bf16 (round to nearest) in HBM --
 * half the bytes every search streams.  A bf16 index scores its rows as the
 * bf16 values widened to fp32 (the reference's arithmetic on those values) and
 * serves k <= 128 (M3G_EUNSUPPORTED above).  No counterpart in the reference,
 * which stores fp32 only (cluster.h:83). */
int m3g_create_ivf_ex(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                      const float* centroids, int64_t nlist, int storage);
/* The list storage of an index (M3G_F32 / M3G_BF16); M3G_ERANGE if unknown. */
int m3g_storage_of(m3g_engine* e, int index_id, int* storage);

/* AsyncEngine::load_cluster (m3_async.cpp:237-260 -> Cluster::rebuild_from,
 * cluster.cpp:152-178): synchronous full replace of one list.  vecs: [n, dim]
 * of dtype M3G_F32 (float) or M3G_BF16 (uint16 bf16 bit patterns); the rows
 * are stored in the index's own storage type. */
int m3g_load_cluster(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                     const void* vecs, int64_t n, int dtype);

/* m3g_load_cluster with the rows already on the engine's device: d_ids [n]
 * int64 and d_vecs [n, dim] of dtype M3G_F32 / M3G_BF16 are device pointers
 * (the zero-host-copy path for data that lives in GPU memory, e.g. a CUDA
 * tensor).  Synchronous. */
int m3g_load_cluster_device(m3g_engine* e, int index_id, int cluster_id, const int64_t* d_ids,
                            const void* d_vecs, int64_t n, int dtype);

/* Every list of index_id replaced at once (Cluster::rebuild_from per list,
 * cluster.cpp:152-178) by the device rows assigned to it: d_assign [n] int32
 * (the list of each row, -1 for none), d_ids [n] int64, d_vecs [n, dim] fp32,
 * all device pointers; a list's rows keep their order.  The same index as
 * m3g_load_cluster list by list, built in one pass over the rows.  Synchronous. */
int m3g_load_lists_device(m3g_engine* e, int index_id, const int32_t* d_assign,
                          const int64_t* d_ids, const float* d_vecs, int64_t n);

/* AsyncEngine::enqueue_insert / enqueue_update / enqueue_delete
 * (m3_async.cpp:123-187; applied by writer threads as Cluster::add_batch /
 * update_batch / erase_batch, cluster.cpp:55-150).  *accepted = 0 when the
 * engine is stopped or the queue is full with block_on_full = 0.
 * Addition without a reference counterpart: an update or delete with
 * cluster_id -1 applies to every list holding the id when the writer reaches it
 * (so callers need not know where an id lives; the reference's backend sends
 * every update and delete to cluster 0); ids held nowhere are ignored, and an
 * update with cluster_id -1 cannot insert (insert_if_absent gives
 * M3G_EINVAL; new ids go through m3g_enqueue_insert_auto). */
int m3g_enqueue_insert(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                       const float* vecs, int64_t n, int* accepted);
int m3g_enqueue_update(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                       const float* vecs, int64_t n, int insert_if_absent, int* accepted);
int m3g_enqueue_delete(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                       int64_t n, int* accepted);

/* AsyncEngine::enqueue_insert_auto (m3_async.cpp:262-313): rows are routed to
 * their nearest centroid on the GPU (bit-exact with IVFIndex::nearest_clusters,
 * m3_index.cpp:243-264) and enqueued as one insert per cluster. */
int m3g_enqueue_insert_auto(m3g_engine* e, int index_id, const int64_t* ids, const float* vecs,
                            int64_t n, int* accepted);

/* AsyncEngine::flush (m3_async.cpp:191-201).  Also reports (and clears) the
 * first error a writer thread hit since the last flush; the reference
 * terminates the process in that case instead. */
int m3g_flush(m3g_engine* e);

/* AsyncEngine::search (m3_async.cpp:205-235 -> IVFIndex::search_nprobe,
 * m3_index.cpp:368-483).  nprobe <= 0 uses the search policy's default_nprobe.
 * Host buffers; synchronous.  An unknown index_id yields empty results, as the
 * reference core does (m3_async.cpp:218-222). */
int m3g_search(m3g_engine* e, int index_id, const float* queries, int64_t nq, int k, int nprobe,
               int64_t* out_ids, float* out_scores, int32_t* out_counts);

/* The same search with device-resident queries and results (device pointers of
 * the engine's device).  With stream == NULL the call is synchronous; with a
 * cudaStream_t it is enqueued on that stream and returns at once (kernel-side
 * errors then surface through m3g_sync_errors). */
int m3g_search_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq, int k,
                      int nprobe, int64_t* d_out_ids, float* d_out_scores, int32_t* d_out_counts,
                      void* stream);
/* Waits for the engine's outstanding device work and reports kernel errors. */
int m3g_sync_errors(m3g_engine* e);

/* IVFIndex::search_on (m3_index.cpp:314-366): search an explicit cluster list
 * (no coarse step); every query probes cluster_ids in the given order. */
int m3g_search_on(m3g_engine* e, int index_id, const int32_t* cluster_ids, int ncluster,
                  const float* queries, int64_t nq, int k, int64_t* out_ids, float* out_scores,
                  int32_t* out_counts);

/* IVFIndex::nearest_clusters (m3_index.cpp:243-264): argmin of the unified
 * score, lowest id on ties, -1 if the index has no lists.  Bit-exact. */
int m3g_nearest_clusters(m3g_engine* e, int index_id, const float* vecs, int64_t n,
                         int32_t* out_cluster);

/* m3g_nearest_clusters on device rows d_vecs [n, dim] fp32, writing
 * d_out_cluster [n] int32 on the device.  Synchronous. */
int m3g_nearest_clusters_device(m3g_engine* e, int index_id, const float* d_vecs, int64_t n,
                                int32_t* d_out_cluster);

/* The top-nprobe centroid selection (IVFIndex::select_nprobe_for_query,
 * m3_index.cpp:492-523) on its own: out_probes[nq, min(nprobe, nlist)]
 * ascending by exact score (ties: lower id). */
int m3g_select_probes(m3g_engine* e, int index_id, const float* queries, int64_t nq, int nprobe,
                      int32_t* out_probes);

/* AsyncEngine::dim_of / metric_of / normalized_of / nlist_of
 * (m3_async.cpp:317-351); an unknown index gives dim 0, COSINE, 1, 0. */
int m3g_info(m3g_engine* e, int index_id, int* dim, int* metric, int* normalized, int* nlist);

/* Cluster::size / live_size (cluster.cpp:45-53). */
int m3g_cluster_size(m3g_engine* e, int index_id, int cluster_id, int64_t* size, int64_t* live);
/* The routing centroids [nlist, dim] (IVFIndex::centroid_ptr, m3_index.cpp:170-175). */
int m3g_get_centroids(m3g_engine* e, int index_id, float* out);
/* The live rows of one list, in row order: their ids [n] and vectors [n, dim]
 * (the data Cluster keeps in ids_ / mat_ with alive_ set, cluster.h:73-86).
 * *out_n is always set to n; with out_ids / out_vecs null only the count is
 * returned, otherwise capacity must be at least n (M3G_EINVAL if not). */
int m3g_get_cluster(m3g_engine* e, int index_id, int cluster_id, int64_t* out_ids,
                    float* out_vecs, int64_t capacity, int64_t* out_n);
/* Native save / load of a whole index: centroids and every list's live rows
 * (writes applied so far; call m3g_flush first for queued ones).  No
 * counterpart in the reference, whose only persistence is the Faiss import
 * (faiss_loader.py).  m3g_load_index replaces index_id (as m3g_create_ivf
 * does) only after the whole file has been read; a missing, truncated or
 * foreign file returns M3G_ERUNTIME / M3G_EINVAL and changes nothing.
 * The file holds an 8-byte magic, int32 dim, metric, normalized, nlist, the
 * centroids, then per list int64 n, int64 ids[n], float vectors[n * dim]. */
int m3g_save_index(m3g_engine* e, int index_id, const char* path);
int m3g_load_index(m3g_engine* e, int index_id, const char* path);
/* rebuild_from_faiss (AgentMemory/M3/faiss_loader.py:24-79): replaces index_id
 * with the contents of a Faiss IndexIVFFlat file (its flat quantizer's
 * centroids, every inverted list's ids and fp32 vectors), read from Faiss's
 * published serialization layout without the faiss package; metric L2 -> L2,
 * inner product -> IP; normalized as given; storage M3G_F32 / M3G_BF16.  Only
 * a plain IndexIVFFlat ("IwFl") with array inverted lists is read
 * (M3G_EUNSUPPORTED otherwise); a missing file is M3G_ERUNTIME, a damaged one
 * M3G_EINVAL / M3G_ERUNTIME, and neither changes the index. */
int m3g_rebuild_from_faiss(m3g_engine* e, int index_id, const char* path, int normalized,
                           int storage);
/* IVFIndex::add_cluster / set_centroid (m3_index.cpp:133-163). */
int m3g_add_cluster(m3g_engine* e, int index_id, const float* centroid, int32_t* out_cluster_id);
int m3g_set_centroid(m3g_engine* e, int index_id, int cluster_id, const float* centroid);
/* IVFIndex::compact_cluster / maintenance_pass (m3_index.cpp:266-312). */
int m3g_compact_cluster(m3g_engine* e, int index_id, int cluster_id);
int m3g_maintenance_pass(m3g_engine* e, int index_id);

/* k-means (no counterpart in the reference, whose centroids always come from
 * the caller): nlist distinct seeded rows as the start, niter rounds of
 * exact-assignment + fp64 mean update, assignment against the final centroids.
 * Host buffers: X[n, dim] -> centroids[nlist, dim], assign[n] (nullable). */
int m3g_kmeans(m3g_engine* e, const float* X, int64_t n, int dim, int metric, int normalized,
               int nlist, int niter, uint64_t seed, float* out_centroids, int32_t* out_assign);
/* Trains centroids on (ids, X) with m3g_kmeans, creates index_id with them
 * (as create_ivf) and loads every row into its list in ascending row order. */
int m3g_train_ivf(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                  const int64_t* ids, const float* X, int64_t n, int nlist, int niter,
                  uint64_t seed, float* out_centroids);
/* Splits one list by 2-means (niter rounds, seeded start rows) into itself and
 * a new list: set_centroid(cluster_id, c0), add_cluster(c1), rows regrouped in
 * list order.  *out_new_cluster = -1 when the list has fewer than 2 live rows. */
int m3g_split_cluster(m3g_engine* e, int index_id, int cluster_id, int niter, uint64_t seed,
                      int32_t* out_new_cluster);

/* One split pass now: every list whose live rows exceed mean_factor times the
 * mean live rows over all lists (taken once, before the first split) is split
 * by m3g_split_cluster in ascending id order, list l with seed + l; new lists
 * take the next ids.  *out_nsplit = lists split.  Built from the primitives
 * the reference's TODO names (set_centroid, add_cluster, rebuild_cluster,
 * m3_index.cpp:133-163, 304-311). */
int m3g_split_oversized(m3g_engine* e, int index_id, double mean_factor, int niter, uint64_t seed,
                        int* out_nsplit);

/* Final merge of a list-sharded search (one shard of the lists per GPU): each
 * shard's answer [nq, k] (as m3g_search_device writes it) gathered into
 * d_scores / d_ids [nshard, nq, k] -> the global top-k [nq, k].  Stands in for
 * the ascending sort that ends IVFIndex::search_nprobe (m3_index.cpp:444-475)
 * when the lists live on several GPUs.  Device pointers; enqueued on `stream`
 * (NULL: synchronous). */
int m3g_merge_shards_device(m3g_engine* e, const float* d_scores, const int64_t* d_ids,
                            int nshard, int64_t nq, int k, int64_t* d_out_ids,
                            float* d_out_scores, int32_t* d_out_counts, void* stream);

/* m3g_merge_shards_device over one gathered buffer, so a single all-gather
 * moves scores and ids: shard s's record starts at d_packed + s * shard_bytes
 * and holds its [nq, k] fp32 scores, then at byte ids_offset its [nq, k] int64
 * ids (shard_bytes, ids_offset and d_packed multiples of 8 bytes). */
int m3g_merge_shards_packed_device(m3g_engine* e, const void* d_packed, int nshard, int64_t nq,
                                   int k, int64_t shard_bytes, int64_t ids_offset,
                                   int64_t* d_out_ids, float* d_out_scores, int32_t* d_out_counts,
                                   void* stream);

/* The pieces of a list-sharded search whose coarse step is sharded as well
 * (each GPU scores only the centroids of the lists it owns).  No single
 * counterpart in the reference: together they restate the coarse selection of
 * IVFIndex::search_nprobe (select_nprobe_for_query, m3_index.cpp:492-523) and
 * its list scan (:390-441) across GPUs.  Device pointers; enqueued on `stream`
 * (NULL: the engine's own stream, waited for).
 *
 * m3g_select_probes_device: m3g_select_probes on device queries [nq, dim],
 * writing [nq, min(nprobe, nlist)] cluster ids ascending by exact score.
 * m3g_select_probe_sets_device: the same sets of cluster ids, each row in an
 * order of the engine's choosing (the same for the same inputs) -- the form the
 * list scan consumes, and cheaper: only the centroids whose place in or out of
 * the top nprobe the GEMM's error bound leaves open are rescored exactly.
 * m3g_probe_scores_device: the exact unified score (unified_score,
 * base.h:22-31, in the reference's fp32 arithmetic) of each pair
 * (query q, centroid d_probes[q, j]), [nq, nprobe]; +inf for ids out of range.
 * m3g_search_probes_device: search_nprobe's scan and merge over the given
 * probes [nq, nprobe] (slot j of query q scans list d_probes[q, j]; -1 skips
 * the slot); outputs as m3g_search_device. */
int m3g_select_probes_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                             int nprobe, int32_t* d_out_probes, void* stream);
int m3g_select_probe_sets_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                                 int nprobe, int32_t* d_out_probes, void* stream);
int m3g_probe_scores_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                            const int32_t* d_probes, int nprobe, float* d_out_scores,
                            void* stream);
int m3g_search_probes_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                             int k, const int32_t* d_probes, int nprobe, int64_t* d_out_ids,
                             float* d_out_scores, int32_t* d_out_counts, void* stream);

/* The top-nprobe selection of m3g_select_probes for callers that cannot
 * allocate GPU memory (a fixed pre-reserved memory pool, a runtime that forbids
 * allocation after start-up, or code that must not trigger the device
 * synchronisation cudaMalloc / cudaFree can cause).  No counterpart in the
 * reference.  Needs no engine: d_queries [nq, dim] and d_centroids [nlist, dim]
 * are device arrays (dim a multiple of 4, 16-byte aligned), d_out_probes
 * [nq, min(nprobe, nlist)] int32 is written ascending by exact score, exactly as
 * m3g_select_probes does.  Its scratch is one fixed 16 MiB device array inside
 * the library (held by every GPU that loads it until the process exits), so
 * nq*nlist + 2*nq + 2*nlist must not exceed 4194304; larger requests return
 * M3G_EUNSUPPORTED.  The first call on a device looks the array up
 * (cudaGetSymbolAddress) and keeps its address for the life of the process;
 * make that call before any stream capture, and do not reset the device
 * (cudaDeviceReset) while the library is loaded.  All calls share the array:
 * calls whose work overlaps on the GPU race.  stream NULL: the work goes to the
 * legacy default stream and the call waits for it (which also waits for other
 * blocking streams); callers that must not synchronise pass a non-blocking
 * stream of their own, on which the call only enqueues. */
int m3g_select_probes_noalloc(const float* d_queries, int64_t nq, const float* d_centroids,
                              int64_t nlist, int dim, int metric, int normalized, int nprobe,
                              int32_t* d_out_probes, void* stream);

/* Test hook for the device-side failure path: with ns > 0, every tensor-core
 * list scan first waits up to ns nanoseconds on a barrier that nothing
 * completes, records the timeout and ends without scanning, so the search
 * returns M3G_ETIMEOUT (the path a real stalled wait takes: every role leaves,
 * copies and MMAs in flight are drained, TMEM is freed, the context stays
 * usable).  0 (the default) turns it off.  No counterpart in the reference. */
int m3g_set_test_wait_limit(m3g_engine* e, uint64_t ns);

/* Row tiles of the list scan (tensor-core path): a list longer than `rows` rows
 * is scanned as tiles of `rows` rows, spread over the SMs, each with its own
 * partial top-k, merged per (query, probe) by the last tile to finish.  rows: a
 * positive multiple of 128; 0 (the default) sizes tiles to about 4 MB of rows,
 * or to 128 rows when a batch has fewer (query, probe) pairs than the GPU has
 * SMs; -1 scans every list whole.  Answers do not depend on it.  No counterpart in
 * the reference (its list loop is serial, m3_index.cpp:426-442). */
int m3g_set_scan_tile_rows(m3g_engine* e, int rows);

/* Per-stage device time of the most recent search (profiling must be on). */
typedef struct {
    float ms_prep, ms_coarse_gemm, ms_select, ms_worklist, ms_scan, ms_merge, ms_total;
    int64_t scan_bytes;     /* sum over distinct probed lists of rows * row bytes */
    int64_t probed_pairs;   /* (query, list) pairs scanned */
    int32_t kernel_launches;
    int32_t nq, nprobe, k;
    int64_t graph_launches;          /* searches replayed as a CUDA graph so far */
    int64_t graph_capture_failures;  /* batch shapes whose capture failed (run directly) */
    int64_t streamed_bytes;  /* rows * row bytes the scan's items stream: a list probed by more
                                queries than one item takes is streamed once per item (the
                                repeats are often served by L2) */
} m3g_profile;
int m3g_set_profiling(m3g_engine* e, int on);
int m3g_last_profile(m3g_engine* e, m3g_profile* out);

#ifdef __cplusplus
}
#endif

#endif /* M3GPU_H */
