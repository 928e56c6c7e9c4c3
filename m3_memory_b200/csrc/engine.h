// engine.h -- host-side engine of libm3gpu: indices with their device list
// arenas, the asynchronous write queue, and the search pipeline.
//
// Mirrors the reference's three layers in one place:
//   m3::Cluster  (AgentMemory/M3/src/cluster.cpp)     -> ListMeta + the arena rows
//   m3::IVFIndex (AgentMemory/M3/src/m3_index.cpp)    -> Index
//   m3::AsyncEngine (AgentMemory/M3/src/m3_async.cpp) -> Engine
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "kernels.h"
#include "m3gpu.h"

namespace m3g {

// An error with its ABI status code.
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] void fail(int code, const std::string& msg);
void check_cuda(cudaError_t e, const char* what);
#define M3G_CK(x) ::m3g::check_cuda((x), #x)

// Sets a device for the scope and restores the caller's afterwards.
class DeviceGuard {
   public:
    explicit DeviceGuard(int dev);
    ~DeviceGuard();

   private:
    int prev_ = -1;
    bool changed_ = false;
};

// Owning device allocation (contents are not preserved by alloc()).
template <class T>
struct DBuf {
    T* p = nullptr;
    size_t n = 0;
    DBuf() = default;
    DBuf(const DBuf&) = delete;
    DBuf& operator=(const DBuf&) = delete;
    ~DBuf() { release(); }
    void alloc(size_t count) {
        release();
        if (count) M3G_CK(cudaMalloc(reinterpret_cast<void**>(&p), count * sizeof(T)));
        n = count;
    }
    // Grows (discarding contents) when fewer than `count` elements are held.
    void ensure(size_t count) {
        if (count > n) alloc(count + count / 4 + 16);
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    void swap(DBuf& o) {
        std::swap(p, o.p);
        std::swap(n, o.n);
    }
};

// One inverted list (m3::Cluster, AgentMemory/M3/include/cluster.h:18-87): its
// segment [off, off + cap) of the arena, of which rows [off, off + len) are in
// use, plus host mirrors of the ids and tombstones and the id -> row map.
struct ListMeta {
    int64_t off = 0, len = 0, cap = 0, live = 0;
    std::vector<int64_t> ids;
    std::vector<uint8_t> alive;
    std::unordered_map<int64_t, int64_t> id2row;
};

struct Index {
    int device = 0;
    int dim = 0, dpad = 0, metric = 0;
    bool normalized = false;
    // list arena row format: fp32 rows of ldr = dpad floats, or (storage bf16)
    // bf16 rows of ldr = max(dim rounded up to 8, 64) elements (16-byte rows, at
    // least one 64-wide TMA box)
    int storage = 0;  // M3G_STORE_FP32 / M3G_STORE_BF16
    int esize = 4, ldr = 0;
    int64_t row_bytes() const { return (int64_t)ldr * esize; }
    // arena row r (as bytes) and its width in fp32 words (for the row copy kernels)
    unsigned char* row_ptr(int64_t r) const {
        return reinterpret_cast<unsigned char*>(vecs.p) + r * row_bytes();
    }
    int row_words() const { return (int)(row_bytes() / 4); }
    bool bf16_rows() const { return esize == 2; }
    std::vector<float> centroids;  // [nlist, dim] host copy (routing centroids)
    std::vector<ListMeta> lists;

    // device: centroids and their norms
    DBuf<float> C, cn, cn2;  // [cap, dpad], [cap], [cap]
    DBuf<__nv_bfloat16> C3;  // [cap, kp] split operand [hi | lo | hi] of the tensor-core GEMM
    size_t c_cap = 0;
    // device: the list arena, [arena_cap] rows of row_bytes() (fp32 or bf16) + per-row
    // ids / tombstones / norms (vecs is sized in fp32 words)
    DBuf<float> vecs, rnorm2;
    DBuf<int64_t> ids;
    DBuf<uint8_t> alive;
    int64_t arena_cap = 0, arena_used = 0;
    // device: per-list metadata, and the lists ordered longest first
    DBuf<int64_t> d_list_off;
    DBuf<int32_t> d_list_len, d_list_order;
    RowMaps maps{};
    bool maps_valid = false;

    std::shared_mutex mu;  // shared: searches; exclusive: every mutation
    cudaStream_t wstream = nullptr;

    Index() = default;
    Index(const Index&) = delete;
    Index& operator=(const Index&) = delete;
    ~Index() {
        if (wstream) cudaStreamDestroy(wstream);
    }
    int nlist() const { return (int)lists.size(); }
};

struct QueuePolicy {
    size_t capacity = 4096, pop_batch_max = 64;
    bool block_on_full = true;
};
struct SearchPolicy {
    int default_nprobe = 8;
    bool parallel_queries = false;
};
struct MaintenancePolicy {
    double period_sec = 1.0;
    size_t split_threshold = 200000;
    double compact_ratio = 0.7;
    bool auto_split = false;
    // > 0: auto_split splits lists with more live rows than this factor times the
    // mean over all lists (split_oversized) instead of the absolute split_threshold
    double split_mean_factor = 0.0;
    int split_niter = 5;  // 2-means rounds per split
};

// cluster_id of an update or delete addressed to every list holding the id
constexpr int kAnyList = -1;

struct WriteOp {
    // kInsertRouted: the rows of one enqueue_insert_auto call with their lists
    // (clusters[i] for row i), applied as one Cluster::add_batch per list
    enum Kind { kInsert, kUpdate, kDelete, kInsertRouted } kind = kInsert;
    int index_id = 0, cluster_id = 0;
    bool insert_if_absent = false;
    std::vector<int64_t> ids;
    std::vector<float> vecs;
    std::vector<int32_t> clusters;
};

// Scratch of the search pipeline, grown on demand and reused across calls.
struct Workspace {
    DBuf<float> Q, qn, qn2, S;
    DBuf<__nv_bfloat16> Q3;  // split query operand [hi | hi | lo]
    DBuf<int32_t> probes, lcount, lstart, lcursor, n_items, item_counter, pair_q, pair_slot;
    DBuf<int32_t> tile_cnt;  // finished row tiles per tiled pair (tensor-core scan)
    DBuf<int32_t> plan;      // work-list planning scratch, 6 per list
    DBuf<ScanItem> items;
    DBuf<float> part_score;
    DBuf<int64_t> part_row;
    DBuf<int64_t> out_ids;
    DBuf<float> out_scores;
    DBuf<int32_t> out_counts;
    DBuf<int> err;
    int* err_host = nullptr;  // pinned copy of err, read after the stream's last sync
    DBuf<unsigned long long> stats;
    cudaStream_t stream = nullptr;
    cudaStream_t last_stream = nullptr;  // stream of the last user (ordered by `done`)
    cudaEvent_t done = nullptr;
    cudaEvent_t ev[8] = {};
    cudaEvent_t legacy = nullptr;  // orders a NULL-stream call after the legacy default stream
    std::mutex mu;
};

class Engine {
   public:
    Engine();
    ~Engine();
    void set_device(int dev);
    int device() const { return device_; }

    void start(int writers, int maint);
    void stop();
    void set_queue_policy(const QueuePolicy& p) { qpol_ = p; }
    void set_search_policy(const SearchPolicy& p) { spol_ = p; }
    // (keeps the split rule of set_split_policy)
    void set_maintenance_policy(const MaintenancePolicy& p) {
        const double f = mpol_.split_mean_factor;
        const int ni = mpol_.split_niter;
        mpol_ = p;
        mpol_.split_mean_factor = f;
        mpol_.split_niter = ni;
    }

    void create_ivf(int index_id, int dim, int metric, bool normalized, const float* C, int64_t nlist,
                    int storage = M3G_STORE_FP32);
    void load_cluster(int index_id, int cid, const int64_t* ids, const float* vecs, int64_t n);
    // the same with device rows: d_vecs [n, dim] fp32 or bf16 bits (dtype), d_ids [n]
    void load_cluster_device(int index_id, int cid, const int64_t* d_ids, const void* d_vecs,
                             int64_t n, int dtype);
    // every list replaced at once by the rows assigned to it (d_assign[i], -1:
    // none), rows of a list in ascending row order; device rows fp32 [n, dim]
    void load_lists_device(int index_id, const int32_t* d_assign, const int64_t* d_ids,
                           const float* d_vecs, int64_t n);
    int storage_of(int index_id);
    bool enqueue(WriteOp&& op);
    bool enqueue_insert_auto(int index_id, const int64_t* ids, const float* vecs, int64_t n);
    void flush();

    // Search entry points.  q_dev: queries are device pointers; out_dev: outputs
    // are device pointers; ext_stream: enqueue on this stream and do not wait.
    void search(int index_id, const float* Q, int64_t nq, int k, int nprobe, bool q_dev,
                int64_t* out_ids, float* out_scores, int32_t* out_counts, bool out_dev,
                cudaStream_t ext_stream);
    void search_on(int index_id, const int32_t* cids, int ncids, const float* Q, int64_t nq, int k,
                   int64_t* out_ids, float* out_scores, int32_t* out_counts);
    void select_probes(int index_id, const float* Q, int64_t nq, int nprobe, int32_t* out);
    // Device-pointer pieces of a list-sharded search whose coarse step is sharded
    // too: the selection over this index's centroids, the exact scores of given
    // (query, centroid) pairs, and a search over caller-given probes (-1: none).
    // Enqueued on ext_stream (null: the engine's stream, waited for).  set_only:
    // each row holds the selected set in no particular order (cheaper: only the
    // centroids near the P-th place are rescored).
    void select_probes_device(int index_id, const float* dQ, int64_t nq, int nprobe,
                              int32_t* d_out, cudaStream_t ext_stream, bool set_only = false);
    void probe_scores_device(int index_id, const float* dQ, int64_t nq, const int32_t* d_probes,
                             int P, float* d_scores, cudaStream_t ext_stream);
    void search_probes_device(int index_id, const float* dQ, int64_t nq, int k,
                              const int32_t* d_probes, int P, int64_t* d_ids, float* d_scores,
                              int32_t* d_counts, cudaStream_t ext_stream);
    void nearest_clusters(int index_id, const float* vecs, int64_t n, int32_t* out,
                          bool on_device = false);
    void sync_errors();

    void info(int index_id, int* dim, int* metric, int* normalized, int* nlist);
    void cluster_size(int index_id, int cid, int64_t* size, int64_t* live);
    void get_centroids(int index_id, float* out);
    // the live rows of a list, in row order; *n_live always, ids / vecs when given
    void get_cluster(int index_id, int cid, int64_t* ids, float* vecs, int64_t cap,
                     int64_t* n_live);
    void save_index(int index_id, const char* path);
    // Faiss IndexIVFFlat file -> index_id (faiss_io.cpp)
    void rebuild_from_faiss(int index_id, const char* path, bool normalized, int storage);
    void load_index(int index_id, const char* path);
    int add_cluster(int index_id, const float* c);
    void set_centroid(int index_id, int cid, const float* c);
    void compact_cluster(int index_id, int cid);
    void maintenance_pass(int index_id);

    void kmeans(const float* X, int64_t n, int dim, int metric, bool normalized, int nlist,
                int niter, uint64_t seed, float* C_out, int32_t* assign_out);
    void train_ivf(int index_id, int dim, int metric, bool normalized, const int64_t* ids,
                   const float* X, int64_t n, int nlist, int niter, uint64_t seed, float* C_out);
    int split_cluster(int index_id, int cid, int niter, uint64_t seed);
    // Splits every list whose live rows exceed mean_factor x the mean live rows over
    // all lists (evaluated once, before the first split), in ascending id order,
    // list l with seed + l.  Returns the number of lists split.
    int split_oversized(int index_id, double mean_factor, int niter, uint64_t seed);
    std::vector<int> oversized_lists(int index_id, double mean_factor);
    void set_split_policy(double mean_factor, int niter) {
        mpol_.split_mean_factor = mean_factor;
        mpol_.split_niter = niter;
    }

    void set_profiling(bool on) { profiling_ = on; }
    void set_test_wait_ns(uint64_t ns) { test_wait_ns_ = ns; }
    // Row tiles of long lists in the tensor-core scan: rows per tile (a positive
    // multiple of 128), 0 for the automatic size (128 rows when a batch has fewer
    // (query, probe) pairs than SMs, else about 4 MB of rows), -1 for none.
    void set_scan_tile_rows(int rows) { scan_tile_rows_ = rows; }
    int scan_tile_rows(const Index& ix, int64_t pairs) const;
    m3g_profile last_profile();

   private:
    std::shared_ptr<Index> find(int index_id) const;
    std::shared_ptr<Index> get(int index_id, const char* who) const;
    void writer_loop();
    void maintenance_loop();
    // applies a run of ops of one index under one exclusive lock, one list
    // metadata refresh at the end; per-op errors are recorded
    void apply_run(std::vector<WriteOp>& ops, size_t b, size_t e);
    void apply_locked(Index& ix, const WriteOp& op);
    void record_error(const std::string& msg, int code);

    // device helpers (callers hold the right index lock)
    void run_search(Index& ix, const float* dQ, int64_t ldq, int64_t nq, int k, int P,
                    const int32_t* fixed_probes, int64_t* d_ids, float* d_scores,
                    int32_t* d_counts, cudaStream_t st, bool profile,
                    bool clear_partials = false);
    // Queries [m, dim] on the device as the index's padded rows: the pointer itself
    // when it already is, else a copy into the workspace.
    const float* stage_queries(const Index& ix, const float* dQ, int64_t m, cudaStream_t st);
    void assign_rows(Index& ix, const float* dX, int64_t ld, const float* xn, const float* xn2,
                     int64_t n, int32_t* d_out, cudaStream_t st);
    // Creates the workspace stream / events on first use; then orders `st` after
    // the previous user of the workspace (blocking only when buffers must grow).
    // scores: the call runs the coarse step (score matrix and split queries).
    void acquire_ws(cudaStream_t st, int64_t nq, int64_t L, int64_t P, int64_t k, int64_t dpad,
                    bool scores = true);

    int device_ = 0;
    int num_sms_ = 148;
    std::unordered_map<int, std::shared_ptr<Index>> indices_;
    mutable std::shared_mutex imu_;

    std::mutex qmu_;
    std::condition_variable q_not_empty_, q_not_full_;
    std::deque<WriteOp> queue_;
    QueuePolicy qpol_;
    SearchPolicy spol_;
    MaintenancePolicy mpol_;
    std::vector<std::thread> writers_, maint_;
    std::atomic<bool> running_{false};
    std::atomic<uint64_t> enqueued_{0}, applied_{0};
    std::mutex maint_mu_;
    std::condition_variable maint_cv_;

    std::mutex err_mu_;
    std::string first_error_;
    int first_error_code_ = 0;

    Workspace ws_;
    std::atomic<bool> profiling_{false};
    uint64_t test_wait_ns_ = 0;  // test hook of the tensor-core scan (0: off)
    int scan_tile_rows_ = 0;     // set_scan_tile_rows
    m3g_profile prof_{};
    bool prof_pending_ = false;
    int64_t prof_row_bytes_ = 0, prof_dim_ = 0;
    int32_t last_launches_ = 0;  // kernels the last search call launched
    cudaStream_t prof_stream_ = nullptr;

    // The search pipeline of one batch shape captured as a CUDA graph (queries in
    // ws_.Q, answers in ws_.out_*), replayed while nothing it baked in changes:
    // every pointer and size its kernels were given is part of the key.
    struct SearchGraph {
        std::vector<uintptr_t> key;
        cudaGraphExec_t exec = nullptr;
    } graph_;
    bool graphs_off_ = false;  // set by M3G_SEARCH_GRAPH=0
    // keys whose capture failed (those shapes run their kernels directly; others
    // keep their graphs), and how graphs were used, for m3g_last_profile
    std::vector<std::vector<uintptr_t>> graph_failed_;
    int64_t graph_launches_ = 0, graph_failures_ = 0;
    std::vector<uintptr_t> graph_key(const Index& ix, int64_t nq, int k, int P) const;
    bool run_search_graph(Index& ix, int64_t nq, int k, int P, cudaStream_t st);
};

// Exact top-nprobe selection with its scratch in a fixed device array
// (noalloc.cu); allocates nothing.
void select_probes_noalloc(const float* dQ, int64_t nq, const float* dC, int64_t nlist, int dim,
                           int metric, int normalized, int nprobe, int32_t* d_out,
                           cudaStream_t st);
size_t noalloc_scratch_floats(int64_t nq, int64_t nlist);

// Seeded sampling shared with the oracle: m distinct indices of [0, n) by a
// partial Fisher-Yates shuffle driven by splitmix64.
void sample_rows(uint64_t seed, int64_t n, int64_t m, int64_t* out);

}  // namespace m3g
