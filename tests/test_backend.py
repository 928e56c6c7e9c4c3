"""The reference-contract memory backend (m3_memory_b200.backend) on CPU, with a
recording stand-in for the engine: key conversion, request routing (updates
and deletes addressed to every list, upserts of unseen keys routed as inserts),
search results keyed by the caller's keys."""
from dataclasses import dataclass
from enum import Enum, auto
from types import SimpleNamespace
from typing import Any, List, Optional

import numpy as np
import pytest

from m3_memory_b200.backend import M3Backend, key_to_id


class Kind(Enum):
    INSERT = auto()
    UPDATE = auto()
    DELETE_IDS = auto()
    DELETE_KNN = auto()
    FLUSH = auto()
    SEARCH = auto()


@dataclass
class Req:
    op: Kind
    index_id: int
    ext_ids: Optional[List[Any]] = None
    vectors: Optional[np.ndarray] = None
    k: Optional[int] = None
    request_id: Optional[str] = None
    nprobe: Optional[int] = None


class FakeEngine:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def rec(*a):
            self.calls.append((name,) + a)
            if name == "search":
                _, q, k, _ = a
                return [[7, 2**62 + 5][:k]] * len(q), [[0.5, 0.75][:k]] * len(q)
            return True
        return rec


Metric = SimpleNamespace(L2="L2", IP="IP", COSINE="COSINE")


def test_key_to_id():
    assert key_to_id(42) == 42 and key_to_id("42") == 42 and key_to_id(" -3 ") == -3
    h = key_to_id("doc-a")
    assert 0 <= h < 2**63 and h == key_to_id("doc-a") and h != key_to_id("doc-b")
    assert key_to_id(str(2**70)) == key_to_id(str(2**70)) < 2**63  # beyond int64: hashed


def test_routing_and_results():
    eng = FakeEngine()
    b = M3Backend(engine=eng, metric_enum=Metric)
    b.create_index(3, SimpleNamespace(dim=4, metric="cosine"))
    assert eng.calls[0] == ("start", 2, 1)
    name, idx, dim, metric, normalized, C = eng.calls[1]
    assert (name, idx, dim, metric, normalized, C.shape) == ("create_ivf", 3, 4, "COSINE", True, (1, 4))
    v = np.ones((2, 4), np.float32)
    r = b.execute([
        Req(Kind.INSERT, 3, ext_ids=[7, "doc-a"], vectors=v),
        Req(Kind.UPDATE, 3, ext_ids=["doc-a", "new"], vectors=v),
        Req(Kind.DELETE_IDS, 3, ext_ids=[7]),
        Req(Kind.SEARCH, 3, vectors=np.zeros((1, 4), np.float32), k=2, request_id="q"),
    ])
    assert (r.upserted, r.updated, r.deleted) == (2, 2, 1)
    names = [c[0] for c in eng.calls[2:]]
    assert names == ["enqueue_insert_auto", "enqueue_update", "enqueue_insert_auto",
                     "enqueue_delete", "flush", "search"]
    upd = eng.calls[3]
    assert upd[2] == -1 and upd[3].tolist() == [key_to_id("doc-a")] and upd[5] is False
    assert eng.calls[4][2].tolist() == [key_to_id("new")]
    assert eng.calls[5][2] == -1 and eng.calls[5][3].tolist() == [7]
    assert eng.calls[7][3:] == (2, 32)  # k, default nprobe
    hits = r.searches["q"][0]
    assert [h.id for h in hits] == ["7", str(2**62 + 5)] and hits[0].score == 0.5
    with pytest.raises(KeyError):
        b.execute([Req(Kind.FLUSH, 9)])
    with pytest.raises(NotImplementedError):
        b.execute([Req(Kind.DELETE_KNN, 3, vectors=v, k=1)])
    b.close()
    assert [c[0] for c in eng.calls[-2:]] == ["flush", "stop"]


def test_search_reports_the_callers_keys():
    eng = FakeEngine()
    b = M3Backend(engine=eng, metric_enum=Metric)
    b.create_index(0, SimpleNamespace(dim=2, metric="ip"))
    b.execute([Req(Kind.INSERT, 0, ext_ids=["doc-a"], vectors=np.ones((1, 2), np.float32))])
    eng.search = lambda idx, q, k, n: ([[key_to_id("doc-a")]], [[0.1]])
    r = b.execute([Req(Kind.SEARCH, 0, vectors=np.ones((1, 2), np.float32), k=1)])
    assert r.searches["req-0"][0][0].id == "doc-a"
