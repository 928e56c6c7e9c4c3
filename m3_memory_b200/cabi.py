"""ctypes binding of libm3gpu's C ABI (include/m3gpu.h).

This is the binding a ctypes user of the engine writes; the parity tests call
the engine through it.  ``Engine`` wraps the handle with numpy conveniences
that keep the ABI's conventions (status codes -> exceptions, padded outputs).
"""
from __future__ import annotations

import ctypes as ct
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libm3gpu.so"

M3G_OK, M3G_EINVAL, M3G_ERANGE, M3G_ERUNTIME, M3G_ECUDA, M3G_ENCCL, M3G_ETIMEOUT, \
    M3G_EUNSUPPORTED = range(8)
L2, IP, COSINE = 0, 1, 2
F32, BF16 = 0, 1  # m3g_dtype: vector element types and list storage


def bf16_bits(x):
    """fp32 values -> their bf16 bit patterns (uint16, round to nearest even)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    r[nan] = 0x7FC0
    return r


def bf16_round(x):
    """fp32 values rounded to bf16 precision (kept as fp32)."""
    return (bf16_bits(x).astype(np.uint32) << 16).view(np.float32)

# Every symbol include/m3gpu.h declares, with (restype, argtypes).
_vp = ct.c_void_p
_i32, _i64, _f64, _sz, _u64 = ct.c_int, ct.c_int64, ct.c_double, ct.c_size_t, ct.c_uint64
_pi = ct.POINTER(ct.c_int)
_pi32 = ct.POINTER(ct.c_int32)
_pi64 = ct.POINTER(ct.c_int64)


class Profile(ct.Structure):
    _fields_ = [("ms_prep", ct.c_float), ("ms_coarse_gemm", ct.c_float),
                ("ms_select", ct.c_float), ("ms_worklist", ct.c_float),
                ("ms_scan", ct.c_float), ("ms_merge", ct.c_float), ("ms_total", ct.c_float),
                ("scan_bytes", ct.c_int64), ("probed_pairs", ct.c_int64),
                ("kernel_launches", ct.c_int32), ("nq", ct.c_int32), ("nprobe", ct.c_int32),
                ("k", ct.c_int32), ("graph_launches", ct.c_int64),
                ("graph_capture_failures", ct.c_int64), ("streamed_bytes", ct.c_int64)]


SIGNATURES = {
    "m3g_last_error": (ct.c_char_p, []),
    "m3g_version": (_i32, []),
    "m3g_engine_create": (_i32, [ct.POINTER(_vp)]),
    "m3g_engine_destroy": (_i32, [_vp]),
    "m3g_set_device": (_i32, [_vp, _i32]),
    "m3g_start": (_i32, [_vp, _i32, _i32]),
    "m3g_stop": (_i32, [_vp]),
    "m3g_set_queue_policy": (_i32, [_vp, _sz, _sz, _i32]),
    "m3g_set_search_policy": (_i32, [_vp, _i32, _i32]),
    "m3g_set_maintenance_policy": (_i32, [_vp, _f64, _sz, _f64, _i32]),
    "m3g_create_ivf": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _i64]),
    "m3g_create_ivf_ex": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _i64, _i32]),
    "m3g_storage_of": (_i32, [_vp, _i32, _pi]),
    "m3g_load_cluster": (_i32, [_vp, _i32, _i32, _vp, _vp, _i64, _i32]),
    "m3g_load_cluster_device": (_i32, [_vp, _i32, _i32, _vp, _vp, _i64, _i32]),
    "m3g_set_split_policy": (_i32, [_vp, _f64, _i32]),
    "m3g_set_test_wait_limit": (_i32, [_vp, _u64]),
    "m3g_set_scan_tile_rows": (_i32, [_vp, _i32]),
    "m3g_load_lists_device": (_i32, [_vp, _i32, _vp, _vp, _vp, _i64]),
    "m3g_merge_shards_packed_device": (_i32, [_vp, _vp, _i32, _i64, _i32, _i64, _i64, _vp, _vp,
                                              _vp, _vp]),
    "m3g_rebuild_from_faiss": (_i32, [_vp, _i32, ct.c_char_p, _i32, _i32]),
    "m3g_split_oversized": (_i32, [_vp, _i32, _f64, _i32, _u64, _pi]),
    "m3g_nearest_clusters_device": (_i32, [_vp, _i32, _vp, _i64, _vp]),
    "m3g_enqueue_insert": (_i32, [_vp, _i32, _i32, _vp, _vp, _i64, _pi]),
    "m3g_enqueue_update": (_i32, [_vp, _i32, _i32, _vp, _vp, _i64, _i32, _pi]),
    "m3g_enqueue_delete": (_i32, [_vp, _i32, _i32, _vp, _i64, _pi]),
    "m3g_enqueue_insert_auto": (_i32, [_vp, _i32, _vp, _vp, _i64, _pi]),
    "m3g_flush": (_i32, [_vp]),
    "m3g_search": (_i32, [_vp, _i32, _vp, _i64, _i32, _i32, _vp, _vp, _vp]),
    "m3g_search_device": (_i32, [_vp, _i32, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp]),
    "m3g_sync_errors": (_i32, [_vp]),
    "m3g_search_on": (_i32, [_vp, _i32, _vp, _i32, _vp, _i64, _i32, _vp, _vp, _vp]),
    "m3g_nearest_clusters": (_i32, [_vp, _i32, _vp, _i64, _vp]),
    "m3g_select_probes": (_i32, [_vp, _i32, _vp, _i64, _i32, _vp]),
    "m3g_info": (_i32, [_vp, _i32, _pi, _pi, _pi, _pi]),
    "m3g_cluster_size": (_i32, [_vp, _i32, _i32, _pi64, _pi64]),
    "m3g_get_centroids": (_i32, [_vp, _i32, _vp]),
    "m3g_add_cluster": (_i32, [_vp, _i32, _vp, _pi32]),
    "m3g_set_centroid": (_i32, [_vp, _i32, _i32, _vp]),
    "m3g_compact_cluster": (_i32, [_vp, _i32, _i32]),
    "m3g_maintenance_pass": (_i32, [_vp, _i32]),
    "m3g_kmeans": (_i32, [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _u64, _vp, _vp]),
    "m3g_train_ivf": (_i32, [_vp, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _i32, _i32, _u64,
                             _vp]),
    "m3g_split_cluster": (_i32, [_vp, _i32, _i32, _i32, _u64, _pi32]),
    "m3g_merge_shards_device": (_i32, [_vp, _vp, _vp, _i32, _i64, _i32, _vp, _vp, _vp, _vp]),
    "m3g_select_probes_device": (_i32, [_vp, _i32, _vp, _i64, _i32, _vp, _vp]),
    "m3g_select_probe_sets_device": (_i32, [_vp, _i32, _vp, _i64, _i32, _vp, _vp]),
    "m3g_probe_scores_device": (_i32, [_vp, _i32, _vp, _i64, _vp, _i32, _vp, _vp]),
    "m3g_search_probes_device": (_i32, [_vp, _i32, _vp, _i64, _i32, _vp, _i32, _vp, _vp, _vp,
                                        _vp]),
    "m3g_get_cluster": (_i32, [_vp, _i32, _i32, _vp, _vp, _i64, _vp]),
    "m3g_save_index": (_i32, [_vp, _i32, ct.c_char_p]),
    "m3g_load_index": (_i32, [_vp, _i32, ct.c_char_p]),
    "m3g_select_probes_noalloc": (_i32, [_vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp,
                                         _vp]),
    "m3g_set_profiling": (_i32, [_vp, _i32]),
    "m3g_last_profile": (_i32, [_vp, ct.POINTER(Profile)]),
}

_lib = None


def lib():
    """Loads libm3gpu.so (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            raise ImportError(f"{LIB_PATH} is missing; build it with "
                              "`python -m m3_memory_b200._build`")
        L = ct.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class M3GError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[m3g status {code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != M3G_OK:
        msg = lib().m3g_last_error().decode()
        if rc == M3G_EINVAL:
            raise ValueError(msg)
        if rc == M3G_ERANGE:
            raise IndexError(msg)
        raise M3GError(rc, msg)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ct.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i64a(a):
    return np.ascontiguousarray(a, dtype=np.int64)


def select_probes_noalloc(q_ptr, nq, c_ptr, nlist, dim, metric, normalized, nprobe, out_ptr,
                          stream=None):
    """m3g_select_probes_noalloc on device pointers (no engine, no allocation)."""
    check(lib().m3g_select_probes_noalloc(ct.c_void_p(q_ptr), nq, ct.c_void_p(c_ptr), nlist, dim,
                                          metric, int(normalized), nprobe, ct.c_void_p(out_ptr),
                                          ct.c_void_p(stream) if stream else None))


class Engine:
    """An m3g_engine handle bound to the current CUDA device."""

    def __init__(self):
        h = ct.c_void_p()
        check(lib().m3g_engine_create(ct.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().m3g_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        # at interpreter exit the module's globals may already be gone: the
        # process is ending and the driver releases the engine's memory
        try:
            self.close()
        except TypeError:
            pass

    # lifecycle / policies
    def start(self, writers=2, maint=1):
        check(lib().m3g_start(self.h, writers, maint))

    def stop(self):
        check(lib().m3g_stop(self.h))

    def set_search_policy(self, default_nprobe=8, parallel_queries=False):
        check(lib().m3g_set_search_policy(self.h, default_nprobe, int(parallel_queries)))

    def set_queue_policy(self, capacity=4096, pop_batch_max=64, block_on_full=True):
        check(lib().m3g_set_queue_policy(self.h, capacity, pop_batch_max, int(block_on_full)))

    def set_maintenance_policy(self, period_sec=1.0, split_threshold=200000, compact_ratio=0.7,
                               auto_split=False):
        check(lib().m3g_set_maintenance_policy(self.h, period_sec, split_threshold,
                                               compact_ratio, int(auto_split)))

    # index
    def create_ivf(self, index_id, dim, metric, normalized, C, storage=F32):
        C = _f32(C).reshape(-1, dim) if np.size(C) else np.zeros((0, dim), np.float32)
        if storage == F32:
            check(lib().m3g_create_ivf(self.h, index_id, dim, metric, int(normalized), _p(C),
                                       C.shape[0]))
        else:
            check(lib().m3g_create_ivf_ex(self.h, index_id, dim, metric, int(normalized), _p(C),
                                          C.shape[0], storage))

    def storage_of(self, index_id):
        s = ct.c_int()
        check(lib().m3g_storage_of(self.h, index_id, ct.byref(s)))
        return s.value

    def load_cluster(self, index_id, cid, ids, vecs):
        """vecs: float32 rows, or uint16 rows of bf16 bit patterns."""
        ids = _i64a(ids)
        if np.asarray(vecs).dtype == np.uint16:
            v = np.ascontiguousarray(vecs, np.uint16)
            check(lib().m3g_load_cluster(self.h, index_id, cid, _p(ids), _p(v), ids.shape[0],
                                         BF16))
        else:
            v = _f32(vecs)
            check(lib().m3g_load_cluster(self.h, index_id, cid, _p(ids), _p(v), ids.shape[0],
                                         F32))

    def load_cluster_device(self, index_id, cid, ids_ptr, vecs_ptr, n, dtype=F32):
        """Device pointers: ids int64 [n], vectors [n, dim] fp32 or bf16 bits."""
        check(lib().m3g_load_cluster_device(self.h, index_id, cid, ct.c_void_p(ids_ptr),
                                            ct.c_void_p(vecs_ptr), n, dtype))

    def load_lists_device(self, index_id, assign_ptr, ids_ptr, vecs_ptr, n):
        """Device pointers: assign int32 [n] (-1: none), ids int64 [n], vectors fp32 [n, dim]."""
        check(lib().m3g_load_lists_device(self.h, index_id, ct.c_void_p(assign_ptr),
                                          ct.c_void_p(ids_ptr), ct.c_void_p(vecs_ptr), n))

    def nearest_clusters_device(self, index_id, vecs_ptr, n, out_ptr):
        check(lib().m3g_nearest_clusters_device(self.h, index_id, ct.c_void_p(vecs_ptr), n,
                                                ct.c_void_p(out_ptr)))

    def enqueue_insert(self, index_id, cid, ids, vecs):
        ids, vecs = _i64a(ids), _f32(vecs)
        ok = ct.c_int()
        check(lib().m3g_enqueue_insert(self.h, index_id, cid, _p(ids), _p(vecs), ids.shape[0],
                                       ct.byref(ok)))
        return bool(ok.value)

    def enqueue_update(self, index_id, cid, ids, vecs, insert_if_absent=False):
        ids, vecs = _i64a(ids), _f32(vecs)
        ok = ct.c_int()
        check(lib().m3g_enqueue_update(self.h, index_id, cid, _p(ids), _p(vecs), ids.shape[0],
                                       int(insert_if_absent), ct.byref(ok)))
        return bool(ok.value)

    def enqueue_delete(self, index_id, cid, ids):
        ids = _i64a(ids)
        ok = ct.c_int()
        check(lib().m3g_enqueue_delete(self.h, index_id, cid, _p(ids), ids.shape[0],
                                       ct.byref(ok)))
        return bool(ok.value)

    def enqueue_insert_auto(self, index_id, ids, vecs):
        ids, vecs = _i64a(ids), _f32(vecs)
        ok = ct.c_int()
        check(lib().m3g_enqueue_insert_auto(self.h, index_id, _p(ids), _p(vecs), ids.shape[0],
                                            ct.byref(ok)))
        return bool(ok.value)

    def flush(self):
        check(lib().m3g_flush(self.h))

    def search(self, index_id, Q, k, nprobe=-1):
        Q = _f32(Q)
        nq = Q.shape[0]
        kk = max(k, 0)
        ids = np.empty((nq, max(kk, 1)), np.int64)
        sc = np.empty((nq, max(kk, 1)), np.float32)
        cnt = np.empty(nq, np.int32)
        check(lib().m3g_search(self.h, index_id, _p(Q), nq, kk, nprobe, _p(ids), _p(sc),
                               _p(cnt)))
        return ids[:, :kk], sc[:, :kk], cnt

    def search_on(self, index_id, cids, Q, k):
        Q = _f32(Q)
        cids = np.ascontiguousarray(cids, np.int32)
        nq = Q.shape[0]
        ids = np.empty((nq, max(k, 1)), np.int64)
        sc = np.empty((nq, max(k, 1)), np.float32)
        cnt = np.empty(nq, np.int32)
        check(lib().m3g_search_on(self.h, index_id, _p(cids), cids.shape[0], _p(Q), nq, k,
                                  _p(ids), _p(sc), _p(cnt)))
        return ids[:, :k], sc[:, :k], cnt

    def nearest_clusters(self, index_id, X):
        X = _f32(X)
        out = np.empty(X.shape[0], np.int32)
        check(lib().m3g_nearest_clusters(self.h, index_id, _p(X), X.shape[0], _p(out)))
        return out

    def select_probes(self, index_id, Q, nprobe):
        Q = _f32(Q)
        L = self.info(index_id)[3]
        P = L if nprobe <= 0 else min(nprobe, L)
        out = np.empty((Q.shape[0], max(P, 1)), np.int32)
        check(lib().m3g_select_probes(self.h, index_id, _p(Q), Q.shape[0], P, _p(out)))
        return out[:, :P]

    def info(self, index_id):
        d, m, n, L = ct.c_int(), ct.c_int(), ct.c_int(), ct.c_int()
        check(lib().m3g_info(self.h, index_id, ct.byref(d), ct.byref(m), ct.byref(n),
                             ct.byref(L)))
        return d.value, m.value, bool(n.value), L.value

    def get_cluster(self, index_id, cid):
        """(ids [n], vectors [n, dim]) of a list's live rows, in row order."""
        n = ct.c_int64()
        check(lib().m3g_get_cluster(self.h, index_id, cid, None, None, 0, ct.byref(n)))
        d = self.info(index_id)[0]
        ids = np.empty(n.value, np.int64)
        vecs = np.empty((n.value, d), np.float32)
        check(lib().m3g_get_cluster(self.h, index_id, cid, _p(ids), _p(vecs), n.value,
                                    ct.byref(n)))
        return ids, vecs

    def rebuild_from_faiss(self, index_id, path, normalized=True, storage=F32):
        check(lib().m3g_rebuild_from_faiss(self.h, index_id, str(path).encode(), int(normalized),
                                           storage))

    def save_index(self, index_id, path):
        check(lib().m3g_save_index(self.h, index_id, str(path).encode()))

    def load_index(self, index_id, path):
        check(lib().m3g_load_index(self.h, index_id, str(path).encode()))

    def cluster_size(self, index_id, cid):
        s, l_ = ct.c_int64(), ct.c_int64()
        check(lib().m3g_cluster_size(self.h, index_id, cid, ct.byref(s), ct.byref(l_)))
        return s.value, l_.value

    def centroids(self, index_id):
        d, _, _, L = self.info(index_id)
        out = np.empty((L, d), np.float32)
        check(lib().m3g_get_centroids(self.h, index_id, _p(out)))
        return out

    def add_cluster(self, index_id, c):
        c = _f32(c)
        out = ct.c_int32()
        check(lib().m3g_add_cluster(self.h, index_id, _p(c), ct.byref(out)))
        return out.value

    def set_centroid(self, index_id, cid, c):
        c = _f32(c)
        check(lib().m3g_set_centroid(self.h, index_id, cid, _p(c)))

    def compact_cluster(self, index_id, cid):
        check(lib().m3g_compact_cluster(self.h, index_id, cid))

    def maintenance_pass(self, index_id):
        check(lib().m3g_maintenance_pass(self.h, index_id))

    def kmeans(self, X, nlist, niter, seed, metric, normalized):
        X = _f32(X)
        n, d = X.shape
        C = np.empty((nlist, d), np.float32)
        a = np.empty(n, np.int32)
        check(lib().m3g_kmeans(self.h, _p(X), n, d, metric, int(normalized), nlist, niter, seed,
                               _p(C), _p(a)))
        return C, a

    def train_ivf(self, index_id, dim, metric, normalized, ids, X, nlist, niter, seed):
        X, ids = _f32(X), _i64a(ids)
        C = np.empty((nlist, dim), np.float32)
        check(lib().m3g_train_ivf(self.h, index_id, dim, metric, int(normalized), _p(ids), _p(X),
                                  X.shape[0], nlist, niter, seed, _p(C)))
        return C

    def set_test_wait_limit(self, ns):
        check(lib().m3g_set_test_wait_limit(self.h, ns))

    def set_scan_tile_rows(self, rows):
        check(lib().m3g_set_scan_tile_rows(self.h, rows))

    def set_split_policy(self, mean_factor=0.0, niter=5):
        check(lib().m3g_set_split_policy(self.h, mean_factor, niter))

    def split_oversized(self, index_id, mean_factor=2.0, niter=5, seed=0):
        out = ct.c_int()
        check(lib().m3g_split_oversized(self.h, index_id, mean_factor, niter, seed,
                                        ct.byref(out)))
        return out.value

    def split_cluster(self, index_id, cid, niter=5, seed=0):
        out = ct.c_int32()
        check(lib().m3g_split_cluster(self.h, index_id, cid, niter, seed, ct.byref(out)))
        return out.value

    def set_profiling(self, on=True):
        check(lib().m3g_set_profiling(self.h, int(on)))

    def last_profile(self) -> dict:
        p = Profile()
        check(lib().m3g_last_profile(self.h, ct.byref(p)))
        return {f: getattr(p, f) for f, _ in Profile._fields_}

    # device fast path (raw device pointers, e.g. torch tensors' data_ptr())
    def search_device(self, index_id, q_ptr, nq, k, nprobe, ids_ptr, scores_ptr, counts_ptr,
                      stream=None):
        check(lib().m3g_search_device(self.h, index_id, ct.c_void_p(q_ptr), nq, k, nprobe,
                                      ct.c_void_p(ids_ptr), ct.c_void_p(scores_ptr),
                                      ct.c_void_p(counts_ptr),
                                      ct.c_void_p(stream) if stream else None))

    def merge_shards_packed_device(self, packed_ptr, nshard, nq, k, shard_bytes, ids_offset,
                                   out_ids_ptr, out_scores_ptr, out_counts_ptr, stream=None):
        check(lib().m3g_merge_shards_packed_device(
            self.h, ct.c_void_p(packed_ptr), nshard, nq, k, shard_bytes, ids_offset,
            ct.c_void_p(out_ids_ptr), ct.c_void_p(out_scores_ptr), ct.c_void_p(out_counts_ptr),
            ct.c_void_p(stream) if stream else None))

    def merge_shards_device(self, scores_ptr, ids_ptr, nshard, nq, k, out_ids_ptr,
                            out_scores_ptr, out_counts_ptr, stream=None):
        check(lib().m3g_merge_shards_device(self.h, ct.c_void_p(scores_ptr), ct.c_void_p(ids_ptr),
                                            nshard, nq, k, ct.c_void_p(out_ids_ptr),
                                            ct.c_void_p(out_scores_ptr),
                                            ct.c_void_p(out_counts_ptr),
                                            ct.c_void_p(stream) if stream else None))

    def select_probes_device(self, index_id, q_ptr, nq, nprobe, out_ptr, stream=None):
        check(lib().m3g_select_probes_device(self.h, index_id, ct.c_void_p(q_ptr), nq, nprobe,
                                             ct.c_void_p(out_ptr),
                                             ct.c_void_p(stream) if stream else None))

    def select_probe_sets_device(self, index_id, q_ptr, nq, nprobe, out_ptr, stream=None):
        """As select_probes_device, each row's ids in an order of the engine's
        choosing: the sets a list scan needs, at less cost."""
        check(lib().m3g_select_probe_sets_device(self.h, index_id, ct.c_void_p(q_ptr), nq,
                                                 nprobe, ct.c_void_p(out_ptr),
                                                 ct.c_void_p(stream) if stream else None))

    def probe_scores_device(self, index_id, q_ptr, nq, probes_ptr, nprobe, out_ptr,
                            stream=None):
        check(lib().m3g_probe_scores_device(self.h, index_id, ct.c_void_p(q_ptr), nq,
                                            ct.c_void_p(probes_ptr), nprobe, ct.c_void_p(out_ptr),
                                            ct.c_void_p(stream) if stream else None))

    def search_probes_device(self, index_id, q_ptr, nq, k, probes_ptr, nprobe, ids_ptr,
                             scores_ptr, counts_ptr, stream=None):
        check(lib().m3g_search_probes_device(self.h, index_id, ct.c_void_p(q_ptr), nq, k,
                                             ct.c_void_p(probes_ptr), nprobe, ct.c_void_p(ids_ptr),
                                             ct.c_void_p(scores_ptr), ct.c_void_p(counts_ptr),
                                             ct.c_void_p(stream) if stream else None))

    def sync_errors(self):
        check(lib().m3g_sync_errors(self.h))
