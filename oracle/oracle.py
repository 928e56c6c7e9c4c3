"""TEST INFRASTRUCTURE (oracle) -- not part of the product.

ctypes front end over the two checkers that ``oracle/Makefile`` builds:

* ``RefIndex`` / ``RefEngine`` drive the reference's own C++ core
  (``m3::IVFIndex``, AgentMemory/M3/include/m3_index.h:18-91, and
  ``m3::AsyncEngine``, AgentMemory/M3/include/m3_async.h:63-169) through
  ``oracle/ref_shim.cpp``.
* ``C`` functions (``score``, ``select_nprobe``, ``search_nprobe``,
  ``nearest_clusters``, ``kmeans_train``, ``split_2means`` ...) call the plain-C
  restatement in ``oracle/m3_oracle.c``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference
arm may import this module.
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
C_LIB = REF_DIR / "liboracle_c.so"
REF_LIB = REF_DIR / "liboracle_ref.so"
# The reference checkout: $M3_REFERENCE_ROOT, else a `reference` directory beside
# this repository's checkout.
REFERENCE_ROOT = Path(os.environ.get("M3_REFERENCE_ROOT", str(HERE.parent.parent / "reference")))

L2, IP, COSINE = 0, 1, 2

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


def build(ref: bool | None = None) -> None:
    """Build the checkers (``make -C oracle``).  The reference core is built only
    when the reference tree is present (``ref=None``) or when asked (``ref=True``)."""
    targets = ["c"]
    if ref or (ref is None and (REFERENCE_ROOT / "AgentMemory/M3/src/base.cpp").is_file()):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_ROOT={REFERENCE_ROOT}", *targets],
                   check=True)


def have_ref() -> bool:
    return REF_LIB.is_file()


_c = None
_r = None


def clib():
    global _c
    if _c is None:
        if not C_LIB.is_file():
            build(ref=False)
        lib = ct.CDLL(str(C_LIB))
        lib.orc_score.restype = ct.c_float
        lib.orc_score.argtypes = [_f32p, _f32p, ct.c_int, ct.c_int, ct.c_int]
        lib.orc_select_nprobe.restype = ct.c_int
        lib.orc_select_nprobe.argtypes = [_f32p, _f32p, ct.c_int, ct.c_int, ct.c_int, ct.c_int,
                                          ct.c_int, _i32p]
        lib.orc_nearest_clusters.restype = None
        lib.orc_nearest_clusters.argtypes = [_f32p, ct.c_int64, _f32p, ct.c_int, ct.c_int,
                                             ct.c_int, ct.c_int, _i32p]
        lib.orc_search_on.restype = ct.c_int
        lib.orc_search_on.argtypes = [_f32p, ct.c_int64, ct.c_int, ct.c_int, ct.c_int, _i64p,
                                      ct.c_int, _f32p, _i64p, ct.c_void_p, _i32p, ct.c_int,
                                      ct.c_int, _i64p, _f32p, _i32p]
        lib.orc_search_nprobe.restype = ct.c_int
        lib.orc_search_nprobe.argtypes = [_f32p, ct.c_int64, ct.c_int, ct.c_int, ct.c_int, _f32p,
                                          ct.c_int, _i64p, _f32p, _i64p, ct.c_void_p, ct.c_int,
                                          ct.c_int, _i64p, _f32p, _i32p, ct.c_void_p]
        lib.orc_sample_rows.restype = ct.c_int
        lib.orc_sample_rows.argtypes = [ct.c_uint64, ct.c_int64, ct.c_int64, _i64p]
        lib.orc_kmeans_update.restype = None
        lib.orc_kmeans_update.argtypes = [_f32p, ct.c_int64, ct.c_int, _i32p, ct.c_int, _f32p]
        lib.orc_kmeans_train.restype = ct.c_int
        lib.orc_kmeans_train.argtypes = [_f32p, ct.c_int64, ct.c_int, ct.c_int, ct.c_int,
                                         ct.c_int, ct.c_int, ct.c_uint64, _f32p, _i32p]
        lib.orc_assign_prefiltered.restype = ct.c_int
        lib.orc_assign_prefiltered.argtypes = [_f32p, _f32p, ct.c_int64, _f32p, ct.c_int,
                                               ct.c_int, ct.c_int, ct.c_int, _f64p, _f64p, _i32p,
                                               ct.POINTER(ct.c_int64)]
        lib.orc_score_pairs.restype = None
        lib.orc_score_pairs.argtypes = [_f32p, _i64p, _f32p, _i32p, ct.c_int64, ct.c_int,
                                        ct.c_int, ct.c_int, _f32p]
        lib.orc_split_2means.restype = ct.c_int
        lib.orc_split_2means.argtypes = [_f32p, ct.c_int64, ct.c_int, ct.c_int, ct.c_int,
                                         ct.c_int, ct.c_uint64, _f32p, _i32p]
        _c = lib
    return _c


def rlib():
    global _r
    if _r is None:
        if not REF_LIB.is_file():
            raise FileNotFoundError(f"{REF_LIB} missing: build it with `make -C oracle ref`")
        lib = ct.CDLL(str(REF_LIB))
        vp = ct.c_void_p
        sig = {
            "ref_last_error": (ct.c_char_p, []),
            "ref_unified_score": (ct.c_float, [_f32p, _f32p, ct.c_int, ct.c_int, ct.c_int]),
            "ref_index_new": (vp, [ct.c_int, ct.c_int, ct.c_int]),
            "ref_index_free": (None, [vp]),
            "ref_set_centroids": (ct.c_int, [vp, _f32p, ct.c_int64]),
            "ref_add_cluster": (ct.c_int, [vp, _f32p, ct.POINTER(ct.c_int32)]),
            "ref_set_centroid": (ct.c_int, [vp, ct.c_int, _f32p]),
            "ref_nlist": (ct.c_int, [vp]),
            "ref_rebuild_cluster": (ct.c_int, [vp, ct.c_int, _i64p, _f32p, ct.c_int64]),
            "ref_add_batch": (ct.c_int, [vp, ct.c_int, _i64p, _f32p, ct.c_int64]),
            "ref_update_batch": (ct.c_int, [vp, ct.c_int, _i64p, _f32p, ct.c_int64, ct.c_int]),
            "ref_erase_batch": (ct.c_int, [vp, ct.c_int, _i64p, ct.c_int64]),
            "ref_compact_cluster": (ct.c_int, [vp, ct.c_int]),
            "ref_maintenance_pass": (ct.c_int, [vp]),
            "ref_nearest_clusters": (ct.c_int, [vp, _f32p, ct.c_int64, _i32p]),
            "ref_search_nprobe": (ct.c_int, [vp, _f32p, ct.c_int64, ct.c_int, ct.c_int, _i64p,
                                             _f32p, _i32p]),
            "ref_search_nprobe_mt": (ct.c_int, [vp, _f32p, ct.c_int64, ct.c_int, ct.c_int,
                                                ct.c_int, _i64p, _f32p, _i32p]),
            "ref_search_on": (ct.c_int, [vp, _i32p, ct.c_int, _f32p, ct.c_int64, ct.c_int, _i64p,
                                         _f32p, _i32p]),
            "ref_engine_new": (vp, []),
            "ref_engine_free": (None, [vp]),
            "ref_engine_start": (ct.c_int, [vp, ct.c_int, ct.c_int]),
            "ref_engine_stop": (ct.c_int, [vp]),
            "ref_engine_create_ivf": (ct.c_int, [vp, ct.c_int, ct.c_int, ct.c_int, ct.c_int,
                                                 _f32p, ct.c_int64]),
            "ref_engine_set_search_policy": (ct.c_int, [vp, ct.c_int]),
            "ref_engine_load_cluster": (ct.c_int, [vp, ct.c_int, ct.c_int, _i64p, _f32p,
                                                   ct.c_int64]),
            "ref_engine_enqueue_insert": (ct.c_int, [vp, ct.c_int, ct.c_int, _i64p, _f32p,
                                                     ct.c_int64, ct.POINTER(ct.c_int)]),
            "ref_engine_enqueue_insert_auto": (ct.c_int, [vp, ct.c_int, _i64p, _f32p, ct.c_int64,
                                                          ct.POINTER(ct.c_int)]),
            "ref_engine_enqueue_update": (ct.c_int, [vp, ct.c_int, ct.c_int, _i64p, _f32p,
                                                     ct.c_int64, ct.c_int,
                                                     ct.POINTER(ct.c_int)]),
            "ref_engine_enqueue_delete": (ct.c_int, [vp, ct.c_int, ct.c_int, _i64p, ct.c_int64,
                                                     ct.POINTER(ct.c_int)]),
            "ref_engine_flush": (ct.c_int, [vp]),
            "ref_engine_search": (ct.c_int, [vp, ct.c_int, _f32p, ct.c_int64, ct.c_int, ct.c_int,
                                             _i64p, _f32p, _i32p]),
            "ref_engine_nlist_of": (ct.c_int, [vp, ct.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _r = lib
    return _r


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i64(a):
    return np.ascontiguousarray(a, dtype=np.int64)


class RefError(RuntimeError):
    pass


def _check(rc):
    if rc != 0:
        raise RefError(f"reference core error {rc}: {rlib().ref_last_error().decode()}")


class RefIndex:
    """The reference's ``m3::IVFIndex`` (AgentMemory/M3/src/m3_index.cpp)."""

    def __init__(self, dim: int, metric: int, normalized: bool):
        self.dim = dim
        self.h = rlib().ref_index_new(dim, metric, int(normalized))
        if not self.h:
            raise RefError(rlib().ref_last_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            rlib().ref_index_free(self.h)
            self.h = None

    def set_centroids(self, C):
        C = _f32(C)
        _check(rlib().ref_set_centroids(self.h, C.reshape(-1), C.shape[0]))

    def add_cluster(self, c) -> int:
        out = ct.c_int32()
        _check(rlib().ref_add_cluster(self.h, _f32(c).reshape(-1), ct.byref(out)))
        return out.value

    def set_centroid(self, cid, c):
        _check(rlib().ref_set_centroid(self.h, cid, _f32(c).reshape(-1)))

    def nlist(self) -> int:
        return rlib().ref_nlist(self.h)

    def rebuild_cluster(self, cid, ids, vecs):
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_rebuild_cluster(self.h, cid, ids, vecs, ids.shape[0]))

    def add_batch(self, cid, ids, vecs):
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_add_batch(self.h, cid, ids, vecs, ids.shape[0]))

    def update_batch(self, cid, ids, vecs, insert_if_absent=False):
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_update_batch(self.h, cid, ids, vecs, ids.shape[0],
                                       int(insert_if_absent)))

    def erase_batch(self, cid, ids):
        ids = _i64(ids)
        _check(rlib().ref_erase_batch(self.h, cid, ids, ids.shape[0]))

    def compact_cluster(self, cid):
        _check(rlib().ref_compact_cluster(self.h, cid))

    def nearest_clusters(self, X):
        X = _f32(X)
        out = np.empty(X.shape[0], np.int32)
        _check(rlib().ref_nearest_clusters(self.h, X.reshape(-1), X.shape[0], out))
        return out

    def search_nprobe(self, Q, k, nprobe, threads=1):
        Q = _f32(Q)
        nq = Q.shape[0]
        ids = np.empty((nq, max(k, 1)), np.int64)
        sc = np.empty((nq, max(k, 1)), np.float32)
        cnt = np.empty(nq, np.int32)
        if threads > 1:
            _check(rlib().ref_search_nprobe_mt(self.h, Q.reshape(-1), nq, k, nprobe, threads,
                                               ids.reshape(-1), sc.reshape(-1), cnt))
        else:
            _check(rlib().ref_search_nprobe(self.h, Q.reshape(-1), nq, k, nprobe,
                                            ids.reshape(-1), sc.reshape(-1), cnt))
        return ids, sc, cnt

    def search_on(self, cids, Q, k):
        Q = _f32(Q)
        cids = np.ascontiguousarray(cids, np.int32)
        nq = Q.shape[0]
        ids = np.empty((nq, max(k, 1)), np.int64)
        sc = np.empty((nq, max(k, 1)), np.float32)
        cnt = np.empty(nq, np.int32)
        _check(rlib().ref_search_on(self.h, cids, cids.shape[0], Q.reshape(-1), nq, k,
                                    ids.reshape(-1), sc.reshape(-1), cnt))
        return ids, sc, cnt


class RefEngine:
    """The reference's ``m3::AsyncEngine`` (AgentMemory/M3/src/m3_async.cpp)."""

    def __init__(self):
        self.h = rlib().ref_engine_new()

    def __del__(self):
        if getattr(self, "h", None):
            rlib().ref_engine_free(self.h)
            self.h = None

    def start(self, writers=2, maint=1):
        _check(rlib().ref_engine_start(self.h, writers, maint))

    def stop(self):
        _check(rlib().ref_engine_stop(self.h))

    def create_ivf(self, index_id, dim, metric, normalized, C):
        C = _f32(C)
        _check(rlib().ref_engine_create_ivf(self.h, index_id, dim, metric, int(normalized),
                                            C.reshape(-1), C.shape[0]))

    def set_search_policy(self, default_nprobe=8):
        _check(rlib().ref_engine_set_search_policy(self.h, default_nprobe))

    def load_cluster(self, index_id, cid, ids, vecs):
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_engine_load_cluster(self.h, index_id, cid, ids, vecs, ids.shape[0]))

    def enqueue_insert(self, index_id, cid, ids, vecs) -> bool:
        ok = ct.c_int()
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_engine_enqueue_insert(self.h, index_id, cid, ids, vecs, ids.shape[0],
                                                ct.byref(ok)))
        return bool(ok.value)

    def enqueue_insert_auto(self, index_id, ids, vecs) -> bool:
        ok = ct.c_int()
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_engine_enqueue_insert_auto(self.h, index_id, ids, vecs, ids.shape[0],
                                                     ct.byref(ok)))
        return bool(ok.value)

    def enqueue_update(self, index_id, cid, ids, vecs, insert_if_absent=False) -> bool:
        ok = ct.c_int()
        ids, vecs = _i64(ids), _f32(vecs).reshape(-1)
        _check(rlib().ref_engine_enqueue_update(self.h, index_id, cid, ids, vecs, ids.shape[0],
                                                int(insert_if_absent), ct.byref(ok)))
        return bool(ok.value)

    def enqueue_delete(self, index_id, cid, ids) -> bool:
        ok = ct.c_int()
        ids = _i64(ids)
        _check(rlib().ref_engine_enqueue_delete(self.h, index_id, cid, ids, ids.shape[0],
                                                ct.byref(ok)))
        return bool(ok.value)

    def flush(self):
        _check(rlib().ref_engine_flush(self.h))

    def search(self, index_id, Q, k, nprobe=-1):
        Q = _f32(Q)
        nq = Q.shape[0]
        ids = np.empty((nq, max(k, 1)), np.int64)
        sc = np.empty((nq, max(k, 1)), np.float32)
        cnt = np.empty(nq, np.int32)
        _check(rlib().ref_engine_search(self.h, index_id, Q.reshape(-1), nq, k, nprobe,
                                        ids.reshape(-1), sc.reshape(-1), cnt))
        return ids, sc, cnt

    def nlist_of(self, index_id) -> int:
        return rlib().ref_engine_nlist_of(self.h, index_id)


# ---------------- C restatement ----------------

class CsrLists:
    """Inverted lists as CSR: rows off[c]..off[c+1]-1 belong to cluster c."""

    def __init__(self, off, vecs, ids, alive=None):
        self.off = _i64(off)
        self.vecs = _f32(vecs)
        self.ids = _i64(ids)
        self.alive = None if alive is None else np.ascontiguousarray(alive, np.uint8)

    @staticmethod
    def from_assign(X, ids, assign, nlist):
        """Lists formed from an assignment, rows kept in ascending row order."""
        assign = np.asarray(assign)
        order = np.argsort(assign, kind="stable")
        counts = np.bincount(assign, minlength=nlist)
        off = np.zeros(nlist + 1, np.int64)
        np.cumsum(counts, out=off[1:])
        return CsrLists(off, X[order], np.asarray(ids)[order])

    def rows(self, c):
        b, e = self.off[c], self.off[c + 1]
        return self.ids[b:e], self.vecs[b:e]

    def to_ref(self, idx: "RefIndex"):
        for c in range(len(self.off) - 1):
            ids, v = self.rows(c)
            if len(ids):
                idx.rebuild_cluster(c, ids, v)
                if self.alive is not None:
                    dead = ids[self.alive[self.off[c]:self.off[c + 1]] == 0]
                    if len(dead):
                        idx.erase_batch(c, dead)


def score(a, b, metric, normalized) -> float:
    a, b = _f32(a), _f32(b)
    return clib().orc_score(a, b, a.shape[0], metric, int(normalized))


def select_nprobe(q, C, metric, normalized, nprobe):
    C = _f32(C)
    out = np.empty(max(nprobe, 1), np.int32)
    m = clib().orc_select_nprobe(_f32(q), C.reshape(-1), C.shape[0], C.shape[1], metric,
                                 int(normalized), nprobe, out)
    return out[:m]


def nearest_clusters(X, C, metric, normalized):
    X, C = _f32(X), _f32(C)
    out = np.empty(X.shape[0], np.int32)
    clib().orc_nearest_clusters(X.reshape(-1), X.shape[0], C.reshape(-1), C.shape[0],
                                X.shape[1], metric, int(normalized), out)
    return out


def search_nprobe(Q, C, lists: CsrLists, metric, normalized, k, nprobe, want_probes=False):
    Q, C = _f32(Q), _f32(C)
    nq, d = Q.shape
    nlist = C.shape[0]
    ids = np.empty((nq, max(k, 1)), np.int64)
    sc = np.empty((nq, max(k, 1)), np.float32)
    cnt = np.empty(nq, np.int32)
    p = nprobe if 0 < nprobe < nlist else nlist
    probes = np.empty((nq, max(p, 1)), np.int32) if want_probes else None
    alive = lists.alive.ctypes.data if lists.alive is not None else None
    clib().orc_search_nprobe(Q.reshape(-1), nq, d, metric, int(normalized), C.reshape(-1),
                             nlist, lists.off, lists.vecs.reshape(-1), lists.ids, alive, k,
                             nprobe, ids.reshape(-1), sc.reshape(-1), cnt,
                             probes.ctypes.data if want_probes else None)
    if want_probes:
        return ids, sc, cnt, probes
    return ids, sc, cnt


def merge_shards(scores, ids):
    """Per-shard answers [nshard, nq, k] (ascending scores, -1 / +inf padding) merged
    into [nq, k]: the k smallest valid (finite, non-NaN) scores by (score, shard,
    position) -- the final ascending sort of IVFIndex::search_nprobe
    (AgentMemory/M3/src/m3_index.cpp:444-475) applied across shards.  Returns
    (ids, scores, counts) padded with -1 / +inf."""
    scores = np.asarray(scores, np.float32)
    ids = np.asarray(ids, np.int64)
    ns, nq, k = scores.shape
    out_ids = np.full((nq, k), -1, np.int64)
    out_sc = np.full((nq, k), np.inf, np.float32)
    cnt = np.zeros(nq, np.int32)
    for q in range(nq):
        s = scores[:, q, :].reshape(-1)  # flat index = shard * k + position
        valid = np.flatnonzero(s < np.inf)  # NaN and +inf compare false
        order = valid[np.lexsort((valid, s[valid]))][:k]
        c = len(order)
        out_sc[q, :c] = s[order]
        out_ids[q, :c] = ids[:, q, :].reshape(-1)[order]
        cnt[q] = c
    return out_ids, out_sc, cnt


def search_on(Q, lists: CsrLists, cids, metric, normalized, k):
    """IVFIndex::search_on restated (explicit cluster list, no coarse step)."""
    Q = _f32(Q)
    nq, d = Q.shape
    cids = np.ascontiguousarray(cids, np.int32)
    ids = np.empty((nq, max(k, 1)), np.int64)
    sc = np.empty((nq, max(k, 1)), np.float32)
    cnt = np.empty(nq, np.int32)
    alive = lists.alive.ctypes.data if lists.alive is not None else None
    clib().orc_search_on(Q.reshape(-1), nq, d, metric, int(normalized), lists.off,
                         len(lists.off) - 1, lists.vecs.reshape(-1), lists.ids, alive, cids,
                         cids.shape[0], k, ids.reshape(-1), sc.reshape(-1), cnt)
    return ids, sc, cnt


def sample_rows(seed, n, m):
    out = np.empty(max(m, 1), np.int64)
    rc = clib().orc_sample_rows(seed, n, m, out)
    if rc:
        raise ValueError("sample_rows: m > n")
    return out[:m]


def kmeans_update(X, assign, C):
    X = _f32(X)
    C = _f32(C).copy()
    clib().orc_kmeans_update(X.reshape(-1), X.shape[0], X.shape[1],
                             np.ascontiguousarray(assign, np.int32), C.shape[0], C.reshape(-1))
    return C


def kmeans_train(X, nlist, niter, seed, metric, normalized):
    X = _f32(X)
    n, d = X.shape
    C = np.empty((nlist, d), np.float32)
    a = np.empty(n, np.int32)
    rc = clib().orc_kmeans_train(X.reshape(-1), n, d, metric, int(normalized), nlist, niter,
                                 seed, C.reshape(-1), a)
    if rc:
        raise ValueError("kmeans_train: nlist must be in [1, n]")
    return C, a


def _norms64(A, block=1 << 16):
    out = np.empty(A.shape[0], np.float64)
    for b in range(0, A.shape[0], block):
        a = A[b:b + block].astype(np.float64)
        out[b:b + block] = np.sqrt(np.einsum("ij,ij->i", a, a))
    return out


def nearest_clusters_fast(X, C, metric, normalized, block=8192, stats=None):
    """``nearest_clusters`` (strict '<', lowest id on exact ties) for large inputs:
    an fp32 BLAS product X C^T proposes, a rigorous error bound keeps every
    centroid that could be the argmin, and those are rescored in the reference's
    own arithmetic (``orc_assign_prefiltered``).  Equal to ``nearest_clusters``
    bit for bit; COSINE without normalisation falls back to it."""
    X, C = _f32(X), _f32(C)
    if metric == COSINE and not normalized:
        return nearest_clusters(X, C, metric, normalized)
    n, d = X.shape
    out = np.empty(n, np.int32)
    if C.shape[0] == 0:
        out[:] = -1
        return out
    cn = _norms64(C)
    Ct = np.ascontiguousarray(C.T)
    resc = ct.c_int64()
    total = 0
    for b in range(0, n, block):
        Xb = X[b:b + block]
        S = np.ascontiguousarray(Xb @ Ct, dtype=np.float32)
        rc = clib().orc_assign_prefiltered(S.reshape(-1), Xb.reshape(-1), Xb.shape[0],
                                           C.reshape(-1), C.shape[0], d, metric,
                                           int(normalized), _norms64(Xb), cn, out[b:b + block],
                                           ct.byref(resc))
        if rc:
            raise ValueError("orc_assign_prefiltered: unsupported metric")
        total += resc.value
    if stats is not None:
        stats["rescored_rows"] = total
    return out


def score_pairs(X, rows, C, cols, metric, normalized):
    """Exact unified scores of the pairs (X[rows[j]], C[cols[j]])."""
    X, C = _f32(X), _f32(C)
    rows = _i64(rows)
    cols = np.ascontiguousarray(cols, np.int32)
    out = np.empty(rows.shape[0], np.float32)
    clib().orc_score_pairs(X.reshape(-1), rows, C.reshape(-1), cols, rows.shape[0], X.shape[1],
                           metric, int(normalized), out)
    return out


def kmeans_train_fast(X, nlist, niter, seed, metric, normalized):
    """``kmeans_train`` with the E-steps done by ``nearest_clusters_fast``: the same
    procedure (seeded init rows, exact assignment, fp64 row-order means, final
    assignment), so the same centroids and assignment bit for bit, at BLAS speed."""
    X = _f32(X)
    n, d = X.shape
    if nlist <= 0 or nlist > n:
        raise ValueError("kmeans_train: nlist must be in [1, n]")
    C = np.ascontiguousarray(X[sample_rows(seed, n, nlist)])
    for _ in range(niter):
        a = nearest_clusters_fast(X, C, metric, normalized)
        C = kmeans_update(X, a, C)
    return C, nearest_clusters_fast(X, C, metric, normalized)


def split_2means(X, niter, seed, metric, normalized):
    X = _f32(X)
    n, d = X.shape
    C = np.empty((2, d), np.float32)
    a = np.empty(n, np.int32)
    rc = clib().orc_split_2means(X.reshape(-1), n, d, metric, int(normalized), niter, seed,
                                 C.reshape(-1), a)
    if rc:
        raise ValueError("split_2means: needs at least 2 rows")
    return C, a


def split_oversized(ref: "RefIndex", lists_rows, mean_factor, niter, seed, metric, normalized):
    """The split pass restated on the reference core: every list with more live rows
    than mean_factor x the mean over all lists (taken before the first split) is
    split, in ascending id order, by the oracle's 2-means (list l seeded seed + l)
    and applied through the reference's own primitives -- set_centroid(l, c0),
    add_cluster(c1), rebuild_cluster of both lists (AgentMemory/M3/src/
    m3_index.cpp:133-163, the steps its TODO at :304-311 names).

    lists_rows: per list a pair (ids int64 [n], vecs float32 [n, d]) of its live
    rows in list order, updated in place (new lists appended).  Returns the new
    lists' ids."""
    L = len(lists_rows)
    total = sum(len(i) for i, _ in lists_rows)
    limit = mean_factor * (total / L) if L else 0.0
    todo = [l for l in range(L) if len(lists_rows[l][0]) > limit]
    new = []
    for l in todo:
        ids, vecs = lists_rows[l]
        if len(ids) < 2:
            continue
        C2, side = split_2means(vecs, niter, seed + l, metric, normalized)
        ref.set_centroid(l, C2[0])
        nid = ref.add_cluster(C2[1])
        a, b = side == 0, side == 1
        lists_rows[l] = (ids[a], vecs[a])
        lists_rows.append((ids[b], vecs[b]))
        ref.rebuild_cluster(l, ids[a], vecs[a])
        ref.rebuild_cluster(nid, ids[b], vecs[b])
        new.append(nid)
    return new
