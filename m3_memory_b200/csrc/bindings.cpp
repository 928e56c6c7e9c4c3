// bindings.cpp -- pybind11 module `_m3_async`: the drop-in replacement of the
// reference's module of the same name (AgentMemory/M3/src/bindings_async.cpp).
//
// Same class and method names, argument names, defaults, shape checks, error
// messages and return types as the reference's AsyncEngine binding
// (bindings_async.cpp:153-588), over the C ABI of libm3gpu (include/m3gpu.h).
// Exceptions: the ABI's status codes map back onto the reference's C++
// exception types as pybind translates them: EINVAL -> ValueError
// (std::invalid_argument), ERANGE -> IndexError (std::out_of_range), everything
// else -> RuntimeError (std::runtime_error).
//
// Additions beyond the reference surface (all new, none shadows a reference
// method): search_into_device (tensor fast path by raw device pointers),
// nearest_clusters, select_probes, search_on, kmeans, train_ivf, split_cluster,
// split_oversized, set_split_policy, rebuild_from_faiss, get_cluster, cluster_size, centroids, save_index, load_index,
// add_cluster, set_centroid, compact_cluster, maintenance_pass, set_device, set_profiling,
// last_profile; and create_ivf's optional `storage` ("fp32" default, or "bf16").
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "m3gpu.h"

namespace py = pybind11;

namespace {

enum class Metric : int { L2 = 0, IP = 1, COSINE = 2 };

void raise_status(int rc) {
    if (rc == M3G_OK) return;
    const std::string msg = m3g_last_error();
    if (rc == M3G_EINVAL) throw std::invalid_argument(msg);
    if (rc == M3G_ERANGE) throw std::out_of_range(msg);
    throw std::runtime_error(msg);
}

using f32arr = py::array_t<float, py::array::c_style | py::array::forcecast>;
using i64arr = py::array_t<int64_t, py::array::c_style | py::array::forcecast>;
using i32arr = py::array_t<int32_t, py::array::c_style | py::array::forcecast>;

class AsyncEngine {
   public:
    AsyncEngine() { raise_status(m3g_engine_create(&e_)); }
    ~AsyncEngine() {
        if (e_) {
            py::gil_scoped_release g;
            m3g_engine_destroy(e_);
        }
    }
    AsyncEngine(const AsyncEngine&) = delete;
    AsyncEngine& operator=(const AsyncEngine&) = delete;

    m3g_engine* h() const { return e_; }

    int dim_of(int index_id) const {
        int d = 0;
        raise_status(m3g_info(e_, index_id, &d, nullptr, nullptr, nullptr));
        return d;
    }
    Metric metric_of(int index_id) const {
        int m = 0;
        raise_status(m3g_info(e_, index_id, nullptr, &m, nullptr, nullptr));
        return (Metric)m;
    }
    bool normalized_of(int index_id) const {
        int n = 0;
        raise_status(m3g_info(e_, index_id, nullptr, nullptr, &n, nullptr));
        return n != 0;
    }
    int nlist_of(int index_id) const {
        int n = 0;
        raise_status(m3g_info(e_, index_id, nullptr, nullptr, nullptr, &n));
        return n;
    }

    // Shape checks of bindings_async.cpp (:257-275 and siblings).
    int check_rows(const char* who, const py::buffer_info& ib, const py::buffer_info& vb,
                   int index_id) const {
        if (ib.ndim != 1) throw std::runtime_error(std::string(who) + "ids must be 1D [N]");
        if (vb.ndim != 2) throw std::runtime_error(std::string(who) + "vectors must be 2D [N, D]");
        if (ib.shape[0] != vb.shape[0])
            throw std::runtime_error(std::string(who) + "ids.size != vectors.N");
        const int d = dim_of(index_id);
        if (d <= 0)
            throw std::runtime_error(std::string(who) +
                                     "unknown index_id (call create_ivf first)");
        if (vb.shape[1] != d)
            throw std::runtime_error(std::string(who) + "vectors dim mismatch, expected " +
                                     std::to_string(d) + ", got " + std::to_string(vb.shape[1]));
        return d;
    }

    py::tuple search(int index_id, f32arr queries, int k, int nprobe) {
        auto b = queries.request();
        if (b.ndim != 2) throw std::runtime_error("queries must be 2D [Q, D]");
        const int d = dim_of(index_id);
        if (d <= 0) throw std::runtime_error("search: unknown index_id (call create_ivf first)");
        if (b.shape[1] != d)
            throw std::runtime_error("search: query dim mismatch, expected " + std::to_string(d) +
                                     ", got " + std::to_string(b.shape[1]));
        const int64_t nq = b.shape[0];
        const int kk = k > 0 ? k : 0;
        std::vector<int64_t> ids((size_t)(nq * kk));
        std::vector<float> sc((size_t)(nq * kk));
        std::vector<int32_t> cnt((size_t)nq);
        int rc;
        {
            py::gil_scoped_release g;
            rc = m3g_search(e_, index_id, static_cast<const float*>(b.ptr), nq, kk, nprobe,
                            ids.data(), sc.data(), cnt.data());
        }
        raise_status(rc);
        py::list out_ids(nq), out_sc(nq);
        for (int64_t q = 0; q < nq; ++q) {
            const int n = cnt[(size_t)q];
            py::list li(n), ls(n);
            for (int j = 0; j < n; ++j) {
                li[j] = py::int_(ids[(size_t)(q * kk + j)]);
                ls[j] = py::float_(sc[(size_t)(q * kk + j)]);
            }
            out_ids[q] = li;
            out_sc[q] = ls;
        }
        return py::make_tuple(out_ids, out_sc);
    }

   private:
    m3g_engine* e_ = nullptr;
};

}  // namespace

PYBIND11_MODULE(_m3_async, m) {
    m.doc() = "M3 Async Engine on B200 (multi-IVF + async writers, CUDA search path)";

    py::enum_<Metric>(m, "Metric")
        .value("L2", Metric::L2)
        .value("IP", Metric::IP)
        .value("COSINE", Metric::COSINE)
        .export_values();

    py::class_<AsyncEngine>(m, "AsyncEngine")
        .def(py::init<>())
        .def(
            "start",
            [](AsyncEngine& e, int writers, int maint) {
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_start(e.h(), writers, maint);
                }
                raise_status(rc);
            },
            py::arg("writer_threads") = 2, py::arg("maintenance_threads") = 1)
        .def("stop",
             [](AsyncEngine& e) {
                 int rc;
                 {
                     py::gil_scoped_release g;
                     rc = m3g_stop(e.h());
                 }
                 raise_status(rc);
             })
        .def(
            "create_ivf",
            [](AsyncEngine& e, int index_id, int dim, Metric metric, bool normalized,
               f32arr centroids, const std::string& storage) {
                auto b = centroids.request();
                if (b.ndim != 2) throw std::runtime_error("centroids must be 2D [nlist, dim]");
                if (b.shape[1] != dim)
                    throw std::runtime_error("centroids dim mismatch: expected " +
                                             std::to_string(dim) + ", got " +
                                             std::to_string(b.shape[1]));
                // storage: "fp32" (the reference's) or "bf16" (rows rounded to bf16 in HBM)
                int st = M3G_STORE_FP32;
                if (storage == "bf16") st = M3G_STORE_BF16;
                else if (storage != "fp32")
                    throw py::value_error("create_ivf: storage must be 'fp32' or 'bf16'");
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_create_ivf_ex(e.h(), index_id, dim, (int)metric, normalized ? 1 : 0,
                                           static_cast<const float*>(b.ptr), b.shape[0], st);
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("dim"), py::arg("metric"), py::arg("normalized"),
            py::arg("centroids"), py::arg("storage") = "fp32")
        .def(
            "set_queue_policy",
            [](AsyncEngine& e, size_t capacity, size_t pop_batch_max, bool block_on_full) {
                raise_status(m3g_set_queue_policy(e.h(), capacity, pop_batch_max,
                                                  block_on_full ? 1 : 0));
            },
            py::arg("capacity") = 4096, py::arg("pop_batch_max") = 64,
            py::arg("block_on_full") = true)
        .def(
            "set_search_policy",
            [](AsyncEngine& e, int default_nprobe, bool parallel_queries) {
                raise_status(m3g_set_search_policy(e.h(), default_nprobe, parallel_queries ? 1 : 0));
            },
            py::arg("default_nprobe") = 8, py::arg("parallel_queries") = false)
        .def(
            "set_maintenance_policy",
            [](AsyncEngine& e, double period_sec, size_t split_threshold, double compact_ratio,
               bool auto_split) {
                raise_status(m3g_set_maintenance_policy(e.h(), period_sec, split_threshold,
                                                        compact_ratio, auto_split ? 1 : 0));
            },
            py::arg("period_sec") = 1.0, py::arg("split_threshold") = 200000,
            py::arg("compact_ratio") = 0.7, py::arg("auto_split") = false)
        .def(
            "enqueue_insert",
            [](AsyncEngine& e, int index_id, int cluster_id, i64arr ids, f32arr vecs) {
                auto ib = ids.request();
                auto vb = vecs.request();
                e.check_rows("enqueue_insert: ", ib, vb, index_id);
                int ok = 0, rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_enqueue_insert(e.h(), index_id, cluster_id,
                                            static_cast<const int64_t*>(ib.ptr),
                                            static_cast<const float*>(vb.ptr), ib.shape[0], &ok);
                }
                raise_status(rc);
                return ok != 0;
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("ids"), py::arg("vectors"))
        .def(
            "enqueue_insert_auto",
            [](AsyncEngine& e, int index_id, i64arr ids, f32arr vecs) {
                auto ib = ids.request();
                auto vb = vecs.request();
                e.check_rows("enqueue_insert_auto: ", ib, vb, index_id);
                int ok = 0, rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_enqueue_insert_auto(e.h(), index_id, static_cast<const int64_t*>(ib.ptr),
                                                 static_cast<const float*>(vb.ptr), ib.shape[0], &ok);
                }
                raise_status(rc);
                return ok != 0;
            },
            py::arg("index_id"), py::arg("ids"), py::arg("vectors"))
        .def(
            "enqueue_update",
            [](AsyncEngine& e, int index_id, int cluster_id, i64arr ids, f32arr vecs,
               bool insert_if_absent) {
                auto ib = ids.request();
                auto vb = vecs.request();
                e.check_rows("enqueue_update: ", ib, vb, index_id);
                int ok = 0, rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_enqueue_update(e.h(), index_id, cluster_id,
                                            static_cast<const int64_t*>(ib.ptr),
                                            static_cast<const float*>(vb.ptr), ib.shape[0],
                                            insert_if_absent ? 1 : 0, &ok);
                }
                raise_status(rc);
                return ok != 0;
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("ids"), py::arg("vectors"),
            py::arg("insert_if_absent") = false)
        .def(
            "enqueue_delete",
            [](AsyncEngine& e, int index_id, int cluster_id, i64arr ids) {
                auto ib = ids.request();
                if (ib.ndim != 1) throw std::runtime_error("ids must be 1D [N]");
                int ok = 0, rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_enqueue_delete(e.h(), index_id, cluster_id,
                                            static_cast<const int64_t*>(ib.ptr), ib.shape[0], &ok);
                }
                raise_status(rc);
                return ok != 0;
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("ids"))
        .def(
            "load_cluster",
            [](AsyncEngine& e, int index_id, int cluster_id, i64arr ids, f32arr vecs) {
                auto ib = ids.request();
                auto vb = vecs.request();
                e.check_rows("load_cluster: ", ib, vb, index_id);
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_load_cluster(e.h(), index_id, cluster_id,
                                          static_cast<const int64_t*>(ib.ptr), vb.ptr,
                                          ib.shape[0], M3G_F32);
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("ids"), py::arg("vectors"))
        .def("flush",
             [](AsyncEngine& e) {
                 int rc;
                 {
                     py::gil_scoped_release g;
                     rc = m3g_flush(e.h());
                 }
                 raise_status(rc);
             })
        .def(
            "search",
            [](AsyncEngine& e, int index_id, f32arr queries, int k) {
                return e.search(index_id, queries, k, -1);
            },
            py::arg("index_id"), py::arg("queries"), py::arg("k"))
        .def(
            "search",
            [](AsyncEngine& e, int index_id, f32arr queries, int k, int nprobe) {
                return e.search(index_id, queries, k, nprobe);
            },
            py::arg("index_id"), py::arg("queries"), py::arg("k"), py::arg("nprobe"))
        .def("dim_of", &AsyncEngine::dim_of)
        .def("metric_of", &AsyncEngine::metric_of)
        .def("normalized_of", &AsyncEngine::normalized_of)
        .def("nlist_of", &AsyncEngine::nlist_of)
        // ---------------- additions ----------------
        .def(
            "search_into_device",
            [](AsyncEngine& e, int index_id, uintptr_t q, int64_t nq, int k, int nprobe,
               uintptr_t out_ids, uintptr_t out_scores, uintptr_t out_counts, uintptr_t stream) {
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_search_device(e.h(), index_id, reinterpret_cast<const float*>(q), nq,
                                           k, nprobe, reinterpret_cast<int64_t*>(out_ids),
                                           reinterpret_cast<float*>(out_scores),
                                           reinterpret_cast<int32_t*>(out_counts),
                                           reinterpret_cast<void*>(stream));
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("queries_ptr"), py::arg("nq"), py::arg("k"),
            py::arg("nprobe"), py::arg("out_ids_ptr"), py::arg("out_scores_ptr"),
            py::arg("out_counts_ptr"), py::arg("stream") = 0)
        .def("sync_errors", [](AsyncEngine& e) {
            int rc;
            {
                py::gil_scoped_release g;
                rc = m3g_sync_errors(e.h());
            }
            raise_status(rc);
        })
        .def(
            "nearest_clusters",
            [](AsyncEngine& e, int index_id, f32arr vecs) {
                auto b = vecs.request();
                if (b.ndim != 2) throw std::runtime_error("vectors must be 2D [N, D]");
                if (b.shape[1] != e.dim_of(index_id))
                    throw std::runtime_error("nearest_clusters: vectors dim mismatch");
                i32arr out(b.shape[0]);
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_nearest_clusters(e.h(), index_id, static_cast<const float*>(b.ptr),
                                              b.shape[0], out.mutable_data());
                }
                raise_status(rc);
                return out;
            },
            py::arg("index_id"), py::arg("vectors"))
        .def(
            "select_probes",
            [](AsyncEngine& e, int index_id, f32arr queries, int nprobe) {
                auto b = queries.request();
                if (b.ndim != 2) throw std::runtime_error("queries must be 2D [Q, D]");
                if (b.shape[1] != e.dim_of(index_id))
                    throw std::runtime_error("select_probes: query dim mismatch");
                const int L = e.nlist_of(index_id);
                const int P = nprobe <= 0 ? L : std::min(nprobe, L);
                i32arr out({(py::ssize_t)b.shape[0], (py::ssize_t)P});
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_select_probes(e.h(), index_id, static_cast<const float*>(b.ptr),
                                           b.shape[0], P, out.mutable_data());
                }
                raise_status(rc);
                return out;
            },
            py::arg("index_id"), py::arg("queries"), py::arg("nprobe"))
        .def(
            "search_on",
            [](AsyncEngine& e, int index_id, i32arr cluster_ids, f32arr queries, int k) {
                auto cb = cluster_ids.request();
                auto b = queries.request();
                if (b.ndim != 2) throw std::runtime_error("queries must be 2D [Q, D]");
                const int64_t nq = b.shape[0];
                const int kk = k > 0 ? k : 0;
                std::vector<int64_t> ids((size_t)(nq * kk));
                std::vector<float> sc((size_t)(nq * kk));
                std::vector<int32_t> cnt((size_t)nq);
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_search_on(e.h(), index_id, static_cast<const int32_t*>(cb.ptr),
                                       (int)cb.size, static_cast<const float*>(b.ptr), nq, kk,
                                       ids.data(), sc.data(), cnt.data());
                }
                raise_status(rc);
                py::list oi(nq), os(nq);
                for (int64_t q = 0; q < nq; ++q) {
                    py::list li(cnt[(size_t)q]), ls(cnt[(size_t)q]);
                    for (int j = 0; j < cnt[(size_t)q]; ++j) {
                        li[j] = py::int_(ids[(size_t)(q * kk + j)]);
                        ls[j] = py::float_(sc[(size_t)(q * kk + j)]);
                    }
                    oi[q] = li;
                    os[q] = ls;
                }
                return py::make_tuple(oi, os);
            },
            py::arg("index_id"), py::arg("cluster_ids"), py::arg("queries"), py::arg("k"))
        .def(
            "kmeans",
            [](AsyncEngine& e, f32arr X, int nlist, int niter, uint64_t seed, Metric metric,
               bool normalized) {
                auto b = X.request();
                if (b.ndim != 2) throw std::runtime_error("X must be 2D [N, D]");
                f32arr C({(py::ssize_t)nlist, (py::ssize_t)b.shape[1]});
                i32arr a(b.shape[0]);
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_kmeans(e.h(), static_cast<const float*>(b.ptr), b.shape[0],
                                    (int)b.shape[1], (int)metric, normalized ? 1 : 0, nlist, niter,
                                    seed, C.mutable_data(), a.mutable_data());
                }
                raise_status(rc);
                return py::make_tuple(C, a);
            },
            py::arg("X"), py::arg("nlist"), py::arg("niter") = 10, py::arg("seed") = 0,
            py::arg("metric") = Metric::L2, py::arg("normalized") = false)
        .def(
            "train_ivf",
            [](AsyncEngine& e, int index_id, int dim, Metric metric, bool normalized, i64arr ids,
               f32arr X, int nlist, int niter, uint64_t seed) {
                auto ib = ids.request();
                auto b = X.request();
                if (b.ndim != 2 || b.shape[1] != dim)
                    throw std::runtime_error("train_ivf: X must be 2D [N, dim]");
                if (ib.ndim != 1 || ib.shape[0] != b.shape[0])
                    throw std::runtime_error("train_ivf: ids.size != X.N");
                f32arr C({(py::ssize_t)nlist, (py::ssize_t)dim});
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_train_ivf(e.h(), index_id, dim, (int)metric, normalized ? 1 : 0,
                                       static_cast<const int64_t*>(ib.ptr),
                                       static_cast<const float*>(b.ptr), b.shape[0], nlist, niter,
                                       seed, C.mutable_data());
                }
                raise_status(rc);
                return C;
            },
            py::arg("index_id"), py::arg("dim"), py::arg("metric"), py::arg("normalized"),
            py::arg("ids"), py::arg("vectors"), py::arg("nlist"), py::arg("niter") = 10,
            py::arg("seed") = 0)
        .def(
            "split_cluster",
            [](AsyncEngine& e, int index_id, int cluster_id, int niter, uint64_t seed) {
                int32_t nid = -1;
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_split_cluster(e.h(), index_id, cluster_id, niter, seed, &nid);
                }
                raise_status(rc);
                return nid;
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("niter") = 5, py::arg("seed") = 0)
        .def(
            "split_oversized",
            [](AsyncEngine& e, int index_id, double mean_factor, int niter, uint64_t seed) {
                int n = 0;
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_split_oversized(e.h(), index_id, mean_factor, niter, seed, &n);
                }
                raise_status(rc);
                return n;
            },
            py::arg("index_id"), py::arg("mean_factor") = 2.0, py::arg("niter") = 5,
            py::arg("seed") = 0)
        .def(
            "set_split_policy",
            [](AsyncEngine& e, double mean_factor, int niter) {
                raise_status(m3g_set_split_policy(e.h(), mean_factor, niter));
            },
            py::arg("mean_factor") = 0.0, py::arg("niter") = 5)
        .def(
            "cluster_size",
            [](AsyncEngine& e, int index_id, int cluster_id) {
                int64_t sz = 0, live = 0;
                raise_status(m3g_cluster_size(e.h(), index_id, cluster_id, &sz, &live));
                return py::make_tuple(sz, live);
            },
            py::arg("index_id"), py::arg("cluster_id"))
        .def(
            "rebuild_from_faiss",
            [](AsyncEngine& e, int index_id, const std::string& path, bool normalized,
               const std::string& storage) {
                int st = M3G_STORE_FP32;
                if (storage == "bf16") st = M3G_STORE_BF16;
                else if (storage != "fp32")
                    throw py::value_error("rebuild_from_faiss: storage must be 'fp32' or 'bf16'");
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_rebuild_from_faiss(e.h(), index_id, path.c_str(), normalized ? 1 : 0,
                                                st);
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("path"), py::arg("normalized") = true,
            py::arg("storage") = "fp32")
        .def(
            "get_cluster",
            [](AsyncEngine& e, int index_id, int cluster_id, bool with_vectors) {
                int64_t n = 0;
                raise_status(m3g_get_cluster(e.h(), index_id, cluster_id, nullptr, nullptr, 0, &n));
                const int d = e.dim_of(index_id);
                py::array_t<int64_t> ids(n);
                py::array_t<float> vecs(std::vector<py::ssize_t>{with_vectors ? n : 0, d});
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_get_cluster(e.h(), index_id, cluster_id, ids.mutable_data(),
                                         with_vectors ? vecs.mutable_data() : nullptr, n, &n);
                }
                raise_status(rc);
                return py::make_tuple(ids, vecs);
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("with_vectors") = true)
        .def(
            "save_index",
            [](AsyncEngine& e, int index_id, const std::string& path) {
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_save_index(e.h(), index_id, path.c_str());
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("path"))
        .def(
            "load_index",
            [](AsyncEngine& e, int index_id, const std::string& path) {
                int rc;
                {
                    py::gil_scoped_release g;
                    rc = m3g_load_index(e.h(), index_id, path.c_str());
                }
                raise_status(rc);
            },
            py::arg("index_id"), py::arg("path"))
        .def(
            "centroids",
            [](AsyncEngine& e, int index_id) {
                const int d = e.dim_of(index_id), L = e.nlist_of(index_id);
                f32arr C({(py::ssize_t)L, (py::ssize_t)(d > 0 ? d : 0)});
                raise_status(m3g_get_centroids(e.h(), index_id, C.mutable_data()));
                return C;
            },
            py::arg("index_id"))
        .def(
            "add_cluster",
            [](AsyncEngine& e, int index_id, f32arr c) {
                auto b = c.request();
                if (b.size != e.dim_of(index_id))
                    throw std::invalid_argument("IVFIndex::add_cluster: centroid dim mismatch");
                int32_t cid = -1;
                raise_status(m3g_add_cluster(e.h(), index_id, static_cast<const float*>(b.ptr), &cid));
                return cid;
            },
            py::arg("index_id"), py::arg("centroid"))
        .def(
            "set_centroid",
            [](AsyncEngine& e, int index_id, int cluster_id, f32arr c) {
                auto b = c.request();
                if (b.size != e.dim_of(index_id))
                    throw std::invalid_argument("IVFIndex::set_centroid: centroid dim mismatch");
                raise_status(
                    m3g_set_centroid(e.h(), index_id, cluster_id, static_cast<const float*>(b.ptr)));
            },
            py::arg("index_id"), py::arg("cluster_id"), py::arg("centroid"))
        .def("compact_cluster",
             [](AsyncEngine& e, int index_id, int cluster_id) {
                 int rc;
                 {
                     py::gil_scoped_release g;
                     rc = m3g_compact_cluster(e.h(), index_id, cluster_id);
                 }
                 raise_status(rc);
             })
        .def("maintenance_pass",
             [](AsyncEngine& e, int index_id) {
                 int rc;
                 {
                     py::gil_scoped_release g;
                     rc = m3g_maintenance_pass(e.h(), index_id);
                 }
                 raise_status(rc);
             })
        .def("set_device",
             [](AsyncEngine& e, int device) { raise_status(m3g_set_device(e.h(), device)); })
        .def("set_profiling",
             [](AsyncEngine& e, bool on) { raise_status(m3g_set_profiling(e.h(), on ? 1 : 0)); })
        .def("last_profile", [](AsyncEngine& e) {
            m3g_profile p{};
            raise_status(m3g_last_profile(e.h(), &p));
            py::dict d;
            d["ms_prep"] = p.ms_prep;
            d["ms_coarse_gemm"] = p.ms_coarse_gemm;
            d["ms_select"] = p.ms_select;
            d["ms_worklist"] = p.ms_worklist;
            d["ms_scan"] = p.ms_scan;
            d["ms_merge"] = p.ms_merge;
            d["ms_total"] = p.ms_total;
            d["scan_bytes"] = p.scan_bytes;
            d["probed_pairs"] = p.probed_pairs;
            d["kernel_launches"] = p.kernel_launches;
            d["nq"] = p.nq;
            d["nprobe"] = p.nprobe;
            d["k"] = p.k;
            d["graph_launches"] = p.graph_launches;
            d["graph_capture_failures"] = p.graph_capture_failures;
            d["streamed_bytes"] = p.streamed_bytes;
            return d;
        });
}
