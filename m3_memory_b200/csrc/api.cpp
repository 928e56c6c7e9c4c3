// api.cpp -- the extern "C" surface of libm3gpu (declared in include/m3gpu.h).
// Every entry point catches C++ exceptions and turns them into an m3g_status
// plus the thread's last-error message.
#include <cstring>
#include <string>

#include "engine.h"
#include "m3gpu.h"

struct m3g_engine {
    m3g::Engine eng;
};

namespace {
thread_local std::string g_last_error;

template <class F>
int guarded(F&& f) {
    try {
        f();
        g_last_error.clear();
        return M3G_OK;
    } catch (const m3g::Error& e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_last_error = "out of host memory";
        return M3G_ERUNTIME;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return M3G_ERUNTIME;
    } catch (...) {
        g_last_error = "unknown error";
        return M3G_ERUNTIME;
    }
}

int bad_handle() {
    g_last_error = "null engine handle";
    return M3G_EINVAL;
}
}  // namespace

#define M3G_ENGINE_OR_FAIL(e) \
    if (!(e)) return bad_handle()

extern "C" {

const char* m3g_last_error(void) { return g_last_error.c_str(); }

int m3g_version(void) { return 20000; }

int m3g_engine_create(m3g_engine** out) {
    if (!out) return bad_handle();
    return guarded([&] { *out = new m3g_engine(); });
}

int m3g_engine_destroy(m3g_engine* e) {
    return guarded([&] { delete e; });
}

int m3g_set_device(m3g_engine* e, int device) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.set_device(device); });
}

int m3g_start(m3g_engine* e, int writer_threads, int maintenance_threads) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.start(writer_threads, maintenance_threads); });
}

int m3g_stop(m3g_engine* e) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.stop(); });
}

int m3g_set_queue_policy(m3g_engine* e, size_t capacity, size_t pop_batch_max, int block_on_full) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        m3g::QueuePolicy p;
        p.capacity = capacity;
        p.pop_batch_max = pop_batch_max;
        p.block_on_full = block_on_full != 0;
        e->eng.set_queue_policy(p);
    });
}

int m3g_set_search_policy(m3g_engine* e, int default_nprobe, int parallel_queries) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        m3g::SearchPolicy p;
        p.default_nprobe = default_nprobe;
        p.parallel_queries = parallel_queries != 0;
        e->eng.set_search_policy(p);
    });
}

int m3g_set_maintenance_policy(m3g_engine* e, double period_sec, size_t split_threshold,
                               double compact_ratio, int auto_split) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        m3g::MaintenancePolicy p;
        p.period_sec = period_sec;
        p.split_threshold = split_threshold;
        p.compact_ratio = compact_ratio;
        p.auto_split = auto_split != 0;
        e->eng.set_maintenance_policy(p);
    });
}

int m3g_set_split_policy(m3g_engine* e, double mean_factor, int niter) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (mean_factor < 0 || niter < 0) m3g::fail(M3G_EINVAL, "set_split_policy: negative value");
        e->eng.set_split_policy(mean_factor, niter);
    });
}

int m3g_split_oversized(m3g_engine* e, int index_id, double mean_factor, int niter, uint64_t seed,
                        int* out_nsplit) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (niter < 0) m3g::fail(M3G_EINVAL, "split_oversized: niter < 0");
        const int n = e->eng.split_oversized(index_id, mean_factor, niter, seed);
        if (out_nsplit) *out_nsplit = n;
    });
}

int m3g_create_ivf(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                   const float* centroids, int64_t nlist) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded(
        [&] { e->eng.create_ivf(index_id, dim, metric, normalized != 0, centroids, nlist); });
}

int m3g_rebuild_from_faiss(m3g_engine* e, int index_id, const char* path, int normalized,
                           int storage) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.rebuild_from_faiss(index_id, path, normalized != 0, storage); });
}

int m3g_set_test_wait_limit(m3g_engine* e, uint64_t ns) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.set_test_wait_ns(ns); });
}

int m3g_set_scan_tile_rows(m3g_engine* e, int rows) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (rows < -1 || (rows > 0 && rows % 128))
            m3g::fail(M3G_EINVAL, "set_scan_tile_rows: rows must be -1, 0 or a positive multiple of 128");
        e->eng.set_scan_tile_rows(rows);
    });
}

int m3g_create_ivf_ex(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                      const float* centroids, int64_t nlist, int storage) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        e->eng.create_ivf(index_id, dim, metric, normalized != 0, centroids, nlist, storage);
    });
}

int m3g_storage_of(m3g_engine* e, int index_id, int* storage) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        const int s = e->eng.storage_of(index_id);
        if (storage) *storage = s;
    });
}

int m3g_load_cluster(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                     const void* vecs, int64_t n, int dtype) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (dtype == M3G_F32) {
            e->eng.load_cluster(index_id, cluster_id, ids, static_cast<const float*>(vecs), n);
            return;
        }
        if (dtype != M3G_BF16) m3g::fail(M3G_EINVAL, "load_cluster: unknown dtype");
        int dim = 0;
        e->eng.info(index_id, &dim, nullptr, nullptr, nullptr);
        if (dim <= 0) m3g::fail(M3G_ERANGE, "AsyncEngine::load_cluster: index not found");
        if (n < 0 || (n > 0 && !vecs))
            m3g::fail(M3G_EINVAL, "AsyncEngine::load_cluster: vecs.size mismatch");
        // bf16 bit patterns widened to fp32 (exact); a bf16 index stores them unchanged
        const uint16_t* b = static_cast<const uint16_t*>(vecs);
        std::vector<float> wide((size_t)(n * dim));
        for (size_t i = 0; i < wide.size(); ++i) {
            const uint32_t u = (uint32_t)b[i] << 16;
            std::memcpy(&wide[i], &u, 4);
        }
        e->eng.load_cluster(index_id, cluster_id, ids, wide.data(), n);
    });
}

namespace {
int enqueue_op(m3g_engine* e, m3g::WriteOp::Kind kind, int index_id, int cluster_id,
               const int64_t* ids, const float* vecs, int64_t n, bool insert_if_absent,
               int* accepted) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (n < 0) m3g::fail(M3G_EINVAL, "enqueue: n < 0");
        int dim = 0;
        e->eng.info(index_id, &dim, nullptr, nullptr, nullptr);
        if (kind != m3g::WriteOp::kDelete && dim <= 0)
            m3g::fail(M3G_ERUNTIME, "enqueue: unknown index_id (call create_ivf first)");
        if (cluster_id == m3g::kAnyList && insert_if_absent)
            m3g::fail(M3G_EINVAL,
                      "enqueue_update: insert_if_absent needs a cluster_id (new ids: "
                      "enqueue_insert_auto)");
        m3g::WriteOp op;
        op.kind = kind;
        op.index_id = index_id;
        op.cluster_id = cluster_id;
        op.insert_if_absent = insert_if_absent;
        if (n > 0) {
            if (!ids) m3g::fail(M3G_EINVAL, "enqueue: ids missing");
            op.ids.assign(ids, ids + n);
            if (kind != m3g::WriteOp::kDelete) {
                if (!vecs) m3g::fail(M3G_EINVAL, "enqueue: vectors missing");
                op.vecs.assign(vecs, vecs + n * (int64_t)dim);
            }
        }
        const bool ok = e->eng.enqueue(std::move(op));
        if (accepted) *accepted = ok ? 1 : 0;
    });
}
}  // namespace

int m3g_enqueue_insert(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                       const float* vecs, int64_t n, int* accepted) {
    return enqueue_op(e, m3g::WriteOp::kInsert, index_id, cluster_id, ids, vecs, n, false,
                      accepted);
}

int m3g_enqueue_update(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids,
                       const float* vecs, int64_t n, int insert_if_absent, int* accepted) {
    return enqueue_op(e, m3g::WriteOp::kUpdate, index_id, cluster_id, ids, vecs, n,
                      insert_if_absent != 0, accepted);
}

int m3g_enqueue_delete(m3g_engine* e, int index_id, int cluster_id, const int64_t* ids, int64_t n,
                       int* accepted) {
    return enqueue_op(e, m3g::WriteOp::kDelete, index_id, cluster_id, ids, nullptr, n, false,
                      accepted);
}

int m3g_enqueue_insert_auto(m3g_engine* e, int index_id, const int64_t* ids, const float* vecs,
                            int64_t n, int* accepted) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        const bool ok = e->eng.enqueue_insert_auto(index_id, ids, vecs, n);
        if (accepted) *accepted = ok ? 1 : 0;
    });
}

int m3g_flush(m3g_engine* e) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.flush(); });
}

int m3g_search(m3g_engine* e, int index_id, const float* queries, int64_t nq, int k, int nprobe,
               int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq > 0 && (!out_counts || (k > 0 && (!out_ids || !out_scores))))
            m3g::fail(M3G_EINVAL, "search: output buffers missing");
        e->eng.search(index_id, queries, nq, k, nprobe, false, out_ids, out_scores, out_counts,
                      false, nullptr);
    });
}

int m3g_search_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq, int k,
                      int nprobe, int64_t* d_out_ids, float* d_out_scores, int32_t* d_out_counts,
                      void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq > 0 && (!d_out_counts || (k > 0 && (!d_out_ids || !d_out_scores))))
            m3g::fail(M3G_EINVAL, "search_device: output buffers missing");
        e->eng.search(index_id, d_queries, nq, k, nprobe, true, d_out_ids, d_out_scores,
                      d_out_counts, true, static_cast<cudaStream_t>(stream));
    });
}

int m3g_sync_errors(m3g_engine* e) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.sync_errors(); });
}

int m3g_search_on(m3g_engine* e, int index_id, const int32_t* cluster_ids, int ncluster,
                  const float* queries, int64_t nq, int k, int64_t* out_ids, float* out_scores,
                  int32_t* out_counts) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        e->eng.search_on(index_id, cluster_ids, ncluster, queries, nq, k, out_ids, out_scores,
                         out_counts);
    });
}

int m3g_nearest_clusters(m3g_engine* e, int index_id, const float* vecs, int64_t n,
                         int32_t* out_cluster) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.nearest_clusters(index_id, vecs, n, out_cluster); });
}

int m3g_load_lists_device(m3g_engine* e, int index_id, const int32_t* d_assign,
                          const int64_t* d_ids, const float* d_vecs, int64_t n) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.load_lists_device(index_id, d_assign, d_ids, d_vecs, n); });
}

int m3g_nearest_clusters_device(m3g_engine* e, int index_id, const float* d_vecs, int64_t n,
                                int32_t* d_out_cluster) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (n > 0 && (!d_vecs || !d_out_cluster))
            m3g::fail(M3G_EINVAL, "nearest_clusters_device: buffers missing");
        e->eng.nearest_clusters(index_id, d_vecs, n, d_out_cluster, true);
    });
}

int m3g_load_cluster_device(m3g_engine* e, int index_id, int cluster_id, const int64_t* d_ids,
                            const void* d_vecs, int64_t n, int dtype) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.load_cluster_device(index_id, cluster_id, d_ids, d_vecs, n, dtype); });
}

int m3g_select_probes(m3g_engine* e, int index_id, const float* queries, int64_t nq, int nprobe,
                      int32_t* out_probes) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.select_probes(index_id, queries, nq, nprobe, out_probes); });
}

int m3g_info(m3g_engine* e, int index_id, int* dim, int* metric, int* normalized, int* nlist) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.info(index_id, dim, metric, normalized, nlist); });
}

int m3g_cluster_size(m3g_engine* e, int index_id, int cluster_id, int64_t* size, int64_t* live) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.cluster_size(index_id, cluster_id, size, live); });
}

int m3g_get_centroids(m3g_engine* e, int index_id, float* out) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.get_centroids(index_id, out); });
}

int m3g_get_cluster(m3g_engine* e, int index_id, int cluster_id, int64_t* out_ids,
                    float* out_vecs, int64_t capacity, int64_t* out_n) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded(
        [&] { e->eng.get_cluster(index_id, cluster_id, out_ids, out_vecs, capacity, out_n); });
}

int m3g_save_index(m3g_engine* e, int index_id, const char* path) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.save_index(index_id, path); });
}

int m3g_load_index(m3g_engine* e, int index_id, const char* path) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.load_index(index_id, path); });
}

int m3g_add_cluster(m3g_engine* e, int index_id, const float* centroid, int32_t* out_cluster_id) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        const int c = e->eng.add_cluster(index_id, centroid);
        if (out_cluster_id) *out_cluster_id = c;
    });
}

int m3g_set_centroid(m3g_engine* e, int index_id, int cluster_id, const float* centroid) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.set_centroid(index_id, cluster_id, centroid); });
}

int m3g_compact_cluster(m3g_engine* e, int index_id, int cluster_id) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.compact_cluster(index_id, cluster_id); });
}

int m3g_maintenance_pass(m3g_engine* e, int index_id) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.maintenance_pass(index_id); });
}

int m3g_kmeans(m3g_engine* e, const float* X, int64_t n, int dim, int metric, int normalized,
               int nlist, int niter, uint64_t seed, float* out_centroids, int32_t* out_assign) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        e->eng.kmeans(X, n, dim, metric, normalized != 0, nlist, niter, seed, out_centroids,
                      out_assign);
    });
}

int m3g_train_ivf(m3g_engine* e, int index_id, int dim, int metric, int normalized,
                  const int64_t* ids, const float* X, int64_t n, int nlist, int niter,
                  uint64_t seed, float* out_centroids) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        e->eng.train_ivf(index_id, dim, metric, normalized != 0, ids, X, n, nlist, niter, seed,
                         out_centroids);
    });
}

int m3g_split_cluster(m3g_engine* e, int index_id, int cluster_id, int niter, uint64_t seed,
                      int32_t* out_new_cluster) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        const int c = e->eng.split_cluster(index_id, cluster_id, niter, seed);
        if (out_new_cluster) *out_new_cluster = c;
    });
}

int m3g_merge_shards_device(m3g_engine* e, const float* d_scores, const int64_t* d_ids,
                            int nshard, int64_t nq, int k, int64_t* d_out_ids,
                            float* d_out_scores, int32_t* d_out_counts, void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nshard <= 0 || nq < 0 || k < 0 || nq > INT32_MAX)
            m3g::fail(M3G_EINVAL, "merge_shards: bad sizes");
        if (nq > 0 && k > 0 && (!d_scores || !d_ids || !d_out_ids || !d_out_scores || !d_out_counts))
            m3g::fail(M3G_EINVAL, "merge_shards: buffers missing");
        m3g::DeviceGuard g(e->eng.device());
        auto st = static_cast<cudaStream_t>(stream);
        M3G_CK(m3g::launch_merge_shards(d_scores, d_ids, nshard, (int)nq, k, d_out_ids,
                                        d_out_scores, d_out_counts, st));
        if (!st) M3G_CK(cudaStreamSynchronize(st));
    });
}

int m3g_merge_shards_packed_device(m3g_engine* e, const void* d_packed, int nshard, int64_t nq,
                                   int k, int64_t shard_bytes, int64_t ids_offset,
                                   int64_t* d_out_ids, float* d_out_scores, int32_t* d_out_counts,
                                   void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nshard <= 0 || nq < 0 || k < 0 || nq > INT32_MAX)
            m3g::fail(M3G_EINVAL, "merge_shards_packed: bad sizes");
        if (nq > 0 && k > 0 && (!d_packed || !d_out_ids || !d_out_scores || !d_out_counts))
            m3g::fail(M3G_EINVAL, "merge_shards_packed: buffers missing");
        if (shard_bytes % 8 || ids_offset % 8 || ids_offset < nq * k * 4 ||
            shard_bytes < ids_offset + nq * k * 8)
            m3g::fail(M3G_EINVAL, "merge_shards_packed: bad record layout");
        m3g::DeviceGuard g(e->eng.device());
        auto st = static_cast<cudaStream_t>(stream);
        M3G_CK(m3g::launch_merge_shards_packed(static_cast<const unsigned char*>(d_packed), nshard,
                                               (int)nq, k, shard_bytes, ids_offset, d_out_ids,
                                               d_out_scores, d_out_counts, st));
        if (!st) M3G_CK(cudaStreamSynchronize(st));
    });
}

int m3g_select_probes_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                             int nprobe, int32_t* d_out_probes, void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq < 0) m3g::fail(M3G_EINVAL, "select_probes_device: nq < 0");
        e->eng.select_probes_device(index_id, d_queries, nq, nprobe, d_out_probes,
                                    static_cast<cudaStream_t>(stream));
    });
}

int m3g_select_probe_sets_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                                 int nprobe, int32_t* d_out_probes, void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq < 0) m3g::fail(M3G_EINVAL, "select_probe_sets_device: nq < 0");
        e->eng.select_probes_device(index_id, d_queries, nq, nprobe, d_out_probes,
                                    static_cast<cudaStream_t>(stream), true);
    });
}

int m3g_probe_scores_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                            const int32_t* d_probes, int nprobe, float* d_out_scores,
                            void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq < 0 || nprobe < 0) m3g::fail(M3G_EINVAL, "probe_scores_device: bad sizes");
        e->eng.probe_scores_device(index_id, d_queries, nq, d_probes, nprobe, d_out_scores,
                                   static_cast<cudaStream_t>(stream));
    });
}

int m3g_search_probes_device(m3g_engine* e, int index_id, const float* d_queries, int64_t nq,
                             int k, const int32_t* d_probes, int nprobe, int64_t* d_out_ids,
                             float* d_out_scores, int32_t* d_out_counts, void* stream) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (nq < 0) m3g::fail(M3G_EINVAL, "search_probes_device: nq < 0");
        e->eng.search_probes_device(index_id, d_queries, nq, k, d_probes, nprobe, d_out_ids,
                                    d_out_scores, d_out_counts, static_cast<cudaStream_t>(stream));
    });
}

int m3g_select_probes_noalloc(const float* d_queries, int64_t nq, const float* d_centroids,
                              int64_t nlist, int dim, int metric, int normalized, int nprobe,
                              int32_t* d_out_probes, void* stream) {
    return guarded([&] {
        m3g::select_probes_noalloc(d_queries, nq, d_centroids, nlist, dim, metric, normalized,
                                   nprobe, d_out_probes, static_cast<cudaStream_t>(stream));
    });
}

int m3g_set_profiling(m3g_engine* e, int on) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] { e->eng.set_profiling(on != 0); });
}

int m3g_last_profile(m3g_engine* e, m3g_profile* out) {
    M3G_ENGINE_OR_FAIL(e);
    return guarded([&] {
        if (!out) m3g::fail(M3G_EINVAL, "last_profile: out missing");
        *out = e->eng.last_profile();
    });
}

}  // extern "C"
