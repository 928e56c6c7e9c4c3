"""A memory backend on this engine with the contract of the reference's
``M3Backend`` (AgentMemory/backend/m3.py:41-208): ``create_index(index_id,
spec)``, ``execute(ops) -> RunResult`` over INSERT / UPDATE / DELETE_IDS / FLUSH /
SEARCH requests, ``close()``.

What differs from that class, all on the caller side of the engine:

* it imports only the engine module (the reference's module also imports a
  multi-level index whose sources do not compile, m3.py:10);
* keys are converted to int64 ids by a function it defines (the reference calls
  an undefined ``_keys_to_int64``, m3.py:134): integers and decimal strings
  that fit int64 are used as they are, any other key maps to a 63-bit BLAKE2b
  hash of its text, and search hits report the key the caller gave;
* updates and deletes reach the lists that hold the ids (cluster_id -1; the
  reference sends them all to cluster 0, m3.py:143,148), and an UPDATE of a key
  this backend has not stored is an insert routed to the nearest list, as the
  reference's insert_if_absent update intends.

The request and result types are the reference's (``AgentMemory.types``) when
that package can be imported, else dataclasses with the same fields; request
kinds are compared by name, so either kind of request works.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Any, Dict, List, Optional

import numpy as np

try:  # the caller's own types, when the reference package is installed
    from AgentMemory.types import RunResult, SearchHit  # type: ignore
except Exception:  # pragma: no cover - depends on the caller's environment
    @dataclass
    class SearchHit:  # noqa: D101 - same fields as AgentMemory.types.SearchHit
        id: str
        score: float
        metadata: Optional[Dict[str, Any]]

    @dataclass
    class RunResult:  # noqa: D101 - same fields as AgentMemory.types.RunResult
        upserted: int
        updated: int
        deleted: int
        searches: Dict[str, List[List[SearchHit]]]

_INT64_MAX = (1 << 63) - 1


def key_to_id(key) -> int:
    """int64 id of a caller key: the integer itself (ints and decimal strings
    within int64), else the low 63 bits of BLAKE2b-64 of the key's text."""
    if isinstance(key, (bool, np.bool_)):
        key = int(key)
    if isinstance(key, (int, np.integer)):
        v = int(key)
        if -_INT64_MAX - 1 <= v <= _INT64_MAX:
            return v
    elif isinstance(key, str):
        s = key.strip()
        if s and (s.isdigit() or (s[0] == "-" and s[1:].isdigit())):
            v = int(s)
            if -_INT64_MAX - 1 <= v <= _INT64_MAX:
                return v
    h = hashlib.blake2b(str(key).encode("utf-8"), digest_size=8).digest()
    return int.from_bytes(h, "little") & _INT64_MAX


def _kind(op) -> str:
    k = getattr(op, "op", None)
    return getattr(k, "name", str(k)).upper()


def _f32_2d(a, err):
    if a is None:
        raise ValueError(err)
    a = np.asarray(a, dtype=np.float32, order="C")
    if a.ndim != 2:
        raise ValueError(err)
    return a


def _metric_name(m) -> str:
    return str(getattr(m, "value", m) or "l2").lower()


class M3Backend:
    """The reference backend's request loop on this engine.  ``engine`` (an
    ``_m3_async.AsyncEngine``-like object) and ``metric_enum`` (its ``Metric``)
    default to this package's pybind module."""

    def __init__(self, autostart: bool = True, writer_threads: int = 2,
                 maintenance_threads: int = 1, engine=None, metric_enum=None,
                 default_nprobe: int = 32):
        if engine is None or metric_enum is None:
            from m3_memory_b200 import _m3_async as m3

            engine = engine if engine is not None else m3.AsyncEngine()
            metric_enum = metric_enum if metric_enum is not None else m3.Metric
        self._eng = engine
        self._metric = metric_enum
        self._autostart = autostart
        self._started = False
        self._writer_threads = writer_threads
        self._maintenance_threads = maintenance_threads
        self._default_nprobe = default_nprobe
        self._indices: set = set()
        self._stored: Dict[int, set] = {}       # index -> ids this backend stored
        self._key_of: Dict[int, Any] = {}       # id -> the caller's key (non-integer keys)

    # ---------- lifecycle (m3.py:65-78) ----------

    def _ensure_started(self):
        if not self._started:
            self._eng.start(self._writer_threads, self._maintenance_threads)
            self._started = True

    def close(self):
        if self._started:
            self._eng.flush()
            self._eng.stop()
            self._started = False

    # ---------- create index (m3.py:82-116) ----------

    def _metric_enum(self, name):
        s = _metric_name(name)
        if s in ("l2", "euclidean"):
            return self._metric.L2
        if s in ("ip", "inner_product", "dot"):
            return self._metric.IP
        if s in ("cos", "cosine"):
            return self._metric.COSINE
        raise ValueError(f"Unsupported metric: {name!r}")

    def create_index(self, index_id: int, spec) -> None:
        if self._autostart:
            self._ensure_started()
        if index_id in self._indices:
            return
        dim = int(spec.dim)
        metric = self._metric_enum(getattr(spec, "metric", "l2"))
        normalized = metric == self._metric.COSINE
        params = getattr(spec, "params", None)
        centroids = params.get("centroids") if params is not None else None
        if centroids is None:
            centroids = np.zeros((1, dim), dtype=np.float32)
        else:
            centroids = np.ascontiguousarray(centroids, dtype=np.float32)
            if centroids.ndim != 2 or centroids.shape[1] != dim:
                raise ValueError("centroids must be [nlist, dim]")
        self._eng.create_ivf(index_id, dim, metric, normalized, centroids)
        self._indices.add(index_id)
        self._stored[index_id] = set()

    # ---------- rebuild from faiss (m3.py:186-198) ----------

    def rebuild_index_from_faiss(self, index_id: int, *, path: str,
                                 normalized: Optional[bool] = None) -> None:
        """The index replaced by a Faiss IndexIVFFlat dump (read by the engine,
        ``m3_memory_b200.faiss_loader.rebuild_from_faiss``); its ids become this
        backend's stored ids, so later UPDATE / DELETE_IDS requests reach them."""
        from m3_memory_b200.faiss_loader import rebuild_from_faiss

        if self._autostart:
            self._ensure_started()
        rebuild_from_faiss(self._eng, index_id=index_id, path=path,
                           normalized=bool(normalized) if normalized is not None else True)
        self._indices.add(index_id)
        stored = self._stored.setdefault(index_id, set())
        stored.clear()
        for c in range(int(self._eng.nlist_of(index_id))):
            ids, _ = self._eng.get_cluster(index_id, c, False)
            stored.update(np.asarray(ids).tolist())

    # ---------- requests (m3.py:120-180) ----------

    def _ids(self, keys, err) -> np.ndarray:
        if keys is None:
            raise ValueError(err)
        out = np.empty(len(keys), np.int64)
        for i, k in enumerate(keys):
            v = key_to_id(k)
            out[i] = v
            if not isinstance(k, (int, np.integer)) and not (isinstance(k, str) and str(v) == k.strip()):
                self._key_of[v] = k
        return out

    def execute(self, ops) -> RunResult:
        if self._autostart:
            self._ensure_started()
        inserted = updated = deleted = 0
        searches: Dict[str, List[List[SearchHit]]] = {}
        for op in ops:
            idx = int(op.index_id)
            if idx not in self._indices:
                raise KeyError(f"M3Backend: index_id {idx} not found. Call create_index() first.")
            kind = _kind(op)
            stored = self._stored[idx]
            if kind == "INSERT":
                ids = self._ids(op.ext_ids, "INSERT requires 'ext_ids'")
                vecs = _f32_2d(op.vectors, "INSERT requires 2D 'vectors'")
                self._eng.enqueue_insert_auto(idx, ids, vecs)
                stored.update(ids.tolist())
                inserted += len(ids)
            elif kind == "UPDATE":
                ids = self._ids(op.ext_ids, "UPDATE requires 'ext_ids'")
                vecs = _f32_2d(op.vectors, "UPDATE requires 2D 'vectors'")
                known = np.array([i in stored for i in ids.tolist()], dtype=bool)
                if known.any():
                    self._eng.enqueue_update(idx, -1, ids[known], vecs[known], False)
                if (~known).any():
                    self._eng.enqueue_insert_auto(idx, ids[~known], vecs[~known])
                    stored.update(ids[~known].tolist())
                updated += len(ids)
            elif kind == "DELETE_IDS":
                ids = self._ids(op.ext_ids, "DELETE_IDS requires 'ext_ids'")
                self._eng.enqueue_delete(idx, -1, ids)
                stored.difference_update(ids.tolist())
                if not any(i in st for st in self._stored.values() for i in ids.tolist()):
                    for i in ids.tolist():
                        self._key_of.pop(i, None)
                deleted += len(ids)
            elif kind == "FLUSH":
                self._eng.flush()
            elif kind == "SEARCH":
                self._eng.flush()
                queries = _f32_2d(op.vectors, "SEARCH requires 2D 'vectors'")
                k = int(op.k or 1)
                nprobe = int(getattr(op, "nprobe", None) or self._default_nprobe)
                out_ids, out_scores = self._eng.search(idx, queries, k, nprobe)
                rid = getattr(op, "request_id", None) or f"req-{len(searches)}"
                searches[rid] = [
                    [SearchHit(id=str(self._key_of.get(int(d), d)), score=float(s), metadata=None)
                     for d, s in zip(row_ids, row_scores)]
                    for row_ids, row_scores in zip(out_ids, out_scores)]
            else:
                raise NotImplementedError(f"Unsupported op: {kind}")
        return RunResult(upserted=inserted, updated=updated, deleted=deleted, searches=searches)
