"""The reference's Python front end, MemoryManagement.run()
(AgentMemory/interface.py:300-416), driven end to end over this repository's
memory backend (m3_memory_b200.backend.M3Backend) with a seeded stub encoder.

The reference package is imported from its own tree ($M3_REFERENCE_ROOT, or a
`reference` directory beside this checkout; skipped where it is absent), with
this repository's modules in the slots of its compiled engine module
(AgentMemory.M3._m3_async and rebuild_from_faiss), which is how a user swaps
the engine in.  The engine itself is a small exact-search stand-in here (this
test runs without a GPU): what is checked is the request path -- queueing,
one-pass encoding, the merged BackendRequests, key conversion, updates and
deletes by id, and search hits carrying the caller's keys back to the
document store."""
import hashlib
import os
import sys
import types
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("M3_REFERENCE_ROOT", str(ROOT.parent / "reference")))


class ExactEngine:
    """The parts of the _m3_async.AsyncEngine contract the backend uses, with
    exact search over every stored row (no lists)."""

    def __init__(self):
        self.ix = {}

    def start(self, *a):
        pass

    def stop(self):
        pass

    def flush(self):
        pass

    def create_ivf(self, index_id, dim, metric, normalized, centroids):
        self.ix[index_id] = {"metric": str(metric), "rows": {}}

    def enqueue_insert_auto(self, index_id, ids, vecs):
        for i, v in zip(ids.tolist(), vecs):
            self.ix[index_id]["rows"][i] = v.copy()
        return True

    def enqueue_update(self, index_id, cid, ids, vecs, insert_if_absent=False):
        rows = self.ix[index_id]["rows"]
        for i, v in zip(ids.tolist(), vecs):
            if i in rows or insert_if_absent:
                rows[i] = v.copy()
        return True

    def enqueue_delete(self, index_id, cid, ids):
        for i in ids.tolist():
            self.ix[index_id]["rows"].pop(i, None)
        return True

    def search(self, index_id, Q, k, nprobe):
        rows = self.ix[index_id]["rows"]
        ids = np.array(list(rows.keys()), np.int64)
        if len(ids) == 0:
            return [[] for _ in Q], [[] for _ in Q]
        X = np.stack(list(rows.values()))
        s = 1.0 - Q @ X.T  # cosine on unit vectors
        out_i, out_s = [], []
        for row in s:
            o = np.argsort(row, kind="stable")[:k]
            out_i.append(ids[o].tolist())
            out_s.append(row[o].tolist())
        return out_i, out_s


class StubEncoder:
    """Seeded unit vectors per text (the same text always maps to the same vector)."""

    dim = 32

    def encode_items(self, items):
        out = []
        for it in items:
            seed = int.from_bytes(hashlib.blake2b(str(it.data).encode(), digest_size=8).digest(),
                                  "little")
            v = np.random.default_rng(seed).standard_normal(self.dim).astype(np.float32)
            out.append(v / np.linalg.norm(v))
        return np.stack(out)


@pytest.fixture()
def reference_front_end(monkeypatch):
    if not (REF / "AgentMemory" / "interface.py").is_file():
        pytest.skip("the reference tree is not present here")
    from m3_memory_b200 import faiss_loader

    # the compiled module's slot, filled as a user swapping the engine in would
    m3pkg = types.ModuleType("AgentMemory.M3")
    m3pkg.__path__ = [str(REF / "AgentMemory" / "M3")]
    fake_async = types.ModuleType("AgentMemory.M3._m3_async")
    fake_async.Metric = types.SimpleNamespace(L2="L2", IP="IP", COSINE="COSINE")
    m3pkg._m3_async = fake_async
    m3pkg.rebuild_from_faiss = faiss_loader.rebuild_from_faiss
    m3pkg.M3MultiLevelIndex = None  # the reference's multi-level index does not compile
    saved = {k: v for k, v in sys.modules.items() if k == "AgentMemory" or k.startswith("AgentMemory.")}
    for k in saved:
        monkeypatch.delitem(sys.modules, k)
    monkeypatch.setitem(sys.modules, "AgentMemory.M3", m3pkg)
    monkeypatch.setitem(sys.modules, "AgentMemory.M3._m3_async", fake_async)
    monkeypatch.syspath_prepend(str(REF))
    import AgentMemory.interface as interface
    import AgentMemory.types as T

    yield interface, T
    for k in [k for k in sys.modules if k == "AgentMemory" or k.startswith("AgentMemory.")]:
        sys.modules.pop(k, None)


def test_memory_management_run_over_the_backend(reference_front_end):
    interface, T = reference_front_end
    from m3_memory_b200.backend import M3Backend

    mm = interface.MemoryManagement(backend="placeholder", encoder=StubEncoder(),
                                    auto_id_strategy="sequential")
    eng = ExactEngine()
    mm.backend = M3Backend(engine=eng, metric_enum=types.SimpleNamespace(
        L2="L2", IP="IP", COSINE="COSINE"))
    mm.create_index("notes", T.Metric.COSINE)
    texts = [f"note number {i}" for i in range(40)]
    mm.add_insert("notes", [T.MemoryItem(id=None, data=t) for t in texts[:30]])
    mm.add_insert("notes", [T.MemoryItem(id=f"doc-{i}", data=t) for i, t in enumerate(texts[30:])])
    r = mm.run()
    assert r.upserted == 40
    # a search for a stored text finds it first, with its payload in the doc store
    mm.add_search("notes", [T.MemoryItem(id=None, data=texts[5]),
                            T.MemoryItem(id=None, data=texts[33])], k=3, request_id="q")
    r = mm.run()
    hits = r.searches["q"]
    assert hits[0][0].score == pytest.approx(0.0, abs=1e-5)
    assert mm.get_doc(hits[0][0].id) == texts[5]
    assert hits[1][0].id == "doc-3" and hits[1][0].score == pytest.approx(0.0, abs=1e-5)
    # update one text in place and delete another, then search again
    mm.add_update("notes", [T.MemoryItem(id="doc-3", data="an entirely different note")])
    mm.add_delete_ids("notes", [hits[0][0].id])
    mm.add_search("notes", [T.MemoryItem(id=None, data=texts[5]),
                            T.MemoryItem(id=None, data="an entirely different note")], k=3,
                  request_id="q2")
    r = mm.run()
    assert (r.updated, r.deleted) == (1, 1)
    h = r.searches["q2"]
    assert hits[0][0].id not in [x.id for x in h[0]]
    assert h[1][0].id == "doc-3" and h[1][0].score == pytest.approx(0.0, abs=1e-5)
    assert len(eng.ix[0]["rows"]) == 39
