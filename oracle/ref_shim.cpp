// ref_shim.cpp -- TEST INFRASTRUCTURE (oracle). Not part of the product.
//
// A small extern "C" shim over the reference's own C++ core (m3::IVFIndex and
// m3::AsyncEngine), compiled together with the reference sources where they lie
// (AgentMemory/M3/src/{base,cluster,m3_index,m3_async}.cpp) by oracle/Makefile.
// The reference's pybind module cannot be used: it also binds MultiLevelIndex,
// whose source (AgentMemory/M3/src/m3_multi_level.cpp:135) does not compile.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
// arm load the resulting liboracle_ref.so. Every function returns 0 on success
// and a negative code on a C++ exception; ref_last_error() gives the message.

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "base.h"
#include "m3_async.h"
#include "m3_index.h"

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return -1;
    } catch (const std::out_of_range& e) {
        g_err = e.what();
        return -2;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -3;
    }
}

// Pads a list-of-lists result into [nq, k] buffers (-1 / +inf) with counts.
void pad_out(const std::vector<std::vector<m3::DocId>>& ids,
             const std::vector<std::vector<float>>& sc, int64_t row0, int k,
             int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    for (size_t q = 0; q < ids.size(); ++q) {
        const int64_t r = row0 + (int64_t)q;
        const int n = (int)ids[q].size();
        out_counts[r] = n;
        for (int j = 0; j < k; ++j) {
            out_ids[r * k + j] = j < n ? ids[q][j] : -1;
            out_scores[r * k + j] =
                j < n ? sc[q][j] : std::numeric_limits<float>::infinity();
        }
    }
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

float ref_unified_score(const float* q, const float* v, int dim, int metric, int normalized) {
    return m3::unified_score(q, v, dim, (m3::Metric)metric, normalized != 0);
}

// ---------------- IVFIndex ----------------

void* ref_index_new(int dim, int metric, int normalized) {
    try {
        return new m3::IVFIndex(dim, (m3::Metric)metric, normalized != 0);
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_index_free(void* h) { delete static_cast<m3::IVFIndex*>(h); }

int ref_set_centroids(void* h, const float* c, int64_t nlist) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<float> v(c, c + nlist * (int64_t)idx->dim());
        idx->set_centroids(v);
    });
}

int ref_add_cluster(void* h, const float* c, int32_t* out_cid) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<float> v(c, c + idx->dim());
        *out_cid = idx->add_cluster(v);
    });
}

int ref_set_centroid(void* h, int cid, const float* c) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<float> v(c, c + idx->dim());
        idx->set_centroid(cid, v);
    });
}

int ref_nlist(void* h) { return static_cast<m3::IVFIndex*>(h)->nlist(); }

int ref_rebuild_cluster(void* h, int cid, const int64_t* ids, const float* vecs, int64_t n) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] { idx->rebuild_cluster(cid, ids, vecs, (size_t)n); });
}

int ref_add_batch(void* h, int cid, const int64_t* ids, const float* vecs, int64_t n) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] { idx->add_batch(cid, ids, vecs, (size_t)n); });
}

int ref_update_batch(void* h, int cid, const int64_t* ids, const float* vecs, int64_t n,
                     int insert_if_absent) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded(
        [&] { idx->update_batch(cid, ids, vecs, (size_t)n, insert_if_absent != 0); });
}

int ref_erase_batch(void* h, int cid, const int64_t* ids, int64_t n) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] { idx->erase_batch(cid, ids, (size_t)n); });
}

int ref_compact_cluster(void* h, int cid) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] { idx->compact_cluster(cid); });
}

int ref_maintenance_pass(void* h) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] { idx->maintenance_pass(); });
}

int ref_nearest_clusters(void* h, const float* vecs, int64_t n, int32_t* out) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<int> o;
        idx->nearest_clusters(vecs, (size_t)n, o);
        for (int64_t i = 0; i < n; ++i) out[i] = o[i];
    });
}

int ref_search_nprobe(void* h, const float* q, int64_t nq, int k, int nprobe,
                      int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<std::vector<m3::DocId>> ids;
        std::vector<std::vector<float>> sc;
        idx->search_nprobe(q, (size_t)nq, k, nprobe, ids, sc);
        pad_out(ids, sc, 0, k, out_ids, out_scores, out_counts);
    });
}

// The query batch split over `threads` std::threads calling search_nprobe
// concurrently (safe: the reference snapshots topology under a shared lock,
// AgentMemory/M3/src/m3_index.cpp:376-382, and scans under per-cluster shared locks).
int ref_search_nprobe_mt(void* h, const float* q, int64_t nq, int k, int nprobe, int threads,
                         int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    if (threads <= 1) return ref_search_nprobe(h, q, nq, k, nprobe, out_ids, out_scores, out_counts);
    std::vector<std::thread> th;
    std::vector<int> rc(threads, 0);
    const int64_t per = (nq + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const int64_t b = t * per, e = std::min<int64_t>(nq, b + per);
        if (b >= e) break;
        th.emplace_back([&, t, b, e] {
            rc[t] = guarded([&] {
                std::vector<std::vector<m3::DocId>> ids;
                std::vector<std::vector<float>> sc;
                idx->search_nprobe(q + b * idx->dim(), (size_t)(e - b), k, nprobe, ids, sc);
                pad_out(ids, sc, b, k, out_ids, out_scores, out_counts);
            });
        });
    }
    for (auto& t : th) t.join();
    for (int r : rc)
        if (r) return r;
    return 0;
}

int ref_search_on(void* h, const int32_t* cids, int ncids, const float* q, int64_t nq, int k,
                  int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    auto* idx = static_cast<m3::IVFIndex*>(h);
    return guarded([&] {
        std::vector<int> c(cids, cids + ncids);
        std::vector<std::vector<m3::DocId>> ids;
        std::vector<std::vector<float>> sc;
        idx->search_on(c, q, (size_t)nq, k, ids, sc);
        pad_out(ids, sc, 0, k, out_ids, out_scores, out_counts);
    });
}

// ---------------- AsyncEngine (engine-level semantics) ----------------

void* ref_engine_new() { return new m3::AsyncEngine(); }
void ref_engine_free(void* h) { delete static_cast<m3::AsyncEngine*>(h); }

int ref_engine_start(void* h, int writers, int maint) {
    return guarded([&] { static_cast<m3::AsyncEngine*>(h)->start(writers, maint); });
}
int ref_engine_stop(void* h) {
    return guarded([&] { static_cast<m3::AsyncEngine*>(h)->stop(); });
}
int ref_engine_create_ivf(void* h, int index_id, int dim, int metric, int normalized,
                          const float* c, int64_t nlist) {
    return guarded([&] {
        std::vector<float> v(c, c + nlist * (int64_t)dim);
        static_cast<m3::AsyncEngine*>(h)->create_ivf(index_id, dim, (m3::Metric)metric,
                                                     normalized != 0, v);
    });
}
int ref_engine_set_search_policy(void* h, int default_nprobe) {
    return guarded([&] {
        m3::AsyncSearchPolicy p;
        p.default_nprobe = default_nprobe;
        static_cast<m3::AsyncEngine*>(h)->set_search_policy(p);
    });
}
int ref_engine_load_cluster(void* h, int index_id, int cid, const int64_t* ids,
                            const float* vecs, int64_t n) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        const int d = e->dim_of(index_id);
        std::vector<m3::DocId> i(ids, ids + n);
        std::vector<float> v(vecs, vecs + n * (int64_t)(d > 0 ? d : 0));
        e->load_cluster(index_id, cid, i, v);
    });
}
int ref_engine_enqueue_insert(void* h, int index_id, int cid, const int64_t* ids,
                              const float* vecs, int64_t n, int* ok) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        m3::InsertOp op;
        op.index_id = index_id;
        op.cluster_id = cid;
        op.ids.assign(ids, ids + n);
        op.vecs.assign(vecs, vecs + n * (int64_t)e->dim_of(index_id));
        *ok = e->enqueue_insert(std::move(op)) ? 1 : 0;
    });
}
int ref_engine_enqueue_insert_auto(void* h, int index_id, const int64_t* ids, const float* vecs,
                                   int64_t n, int* ok) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        std::vector<m3::DocId> i(ids, ids + n);
        std::vector<float> v(vecs, vecs + n * (int64_t)e->dim_of(index_id));
        *ok = e->enqueue_insert_auto(index_id, i, v) ? 1 : 0;
    });
}
int ref_engine_enqueue_update(void* h, int index_id, int cid, const int64_t* ids,
                              const float* vecs, int64_t n, int insert_if_absent, int* ok) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        m3::UpdateOp op;
        op.index_id = index_id;
        op.cluster_id = cid;
        op.insert_if_absent = insert_if_absent != 0;
        op.ids.assign(ids, ids + n);
        op.vecs.assign(vecs, vecs + n * (int64_t)e->dim_of(index_id));
        *ok = e->enqueue_update(std::move(op)) ? 1 : 0;
    });
}
int ref_engine_enqueue_delete(void* h, int index_id, int cid, const int64_t* ids, int64_t n,
                              int* ok) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        m3::DeleteOp op;
        op.index_id = index_id;
        op.cluster_id = cid;
        op.ids.assign(ids, ids + n);
        *ok = e->enqueue_delete(std::move(op)) ? 1 : 0;
    });
}
int ref_engine_flush(void* h) {
    return guarded([&] { static_cast<m3::AsyncEngine*>(h)->flush(); });
}
int ref_engine_search(void* h, int index_id, const float* q, int64_t nq, int k, int nprobe,
                      int64_t* out_ids, float* out_scores, int32_t* out_counts) {
    auto* e = static_cast<m3::AsyncEngine*>(h);
    return guarded([&] {
        std::vector<std::vector<m3::DocId>> ids;
        std::vector<std::vector<float>> sc;
        e->search(index_id, q, (size_t)nq, k, nprobe, ids, sc);
        pad_out(ids, sc, 0, k, out_ids, out_scores, out_counts);
    });
}
int ref_engine_nlist_of(void* h, int index_id) {
    return static_cast<m3::AsyncEngine*>(h)->nlist_of(index_id);
}

}  // extern "C"
