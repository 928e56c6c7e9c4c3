"""The reference-contract memory backend on the real engine (pybind module):
string keys in, string keys out; deletes and updates reach the lists that
hold the keys."""
from types import SimpleNamespace

import numpy as np
import pytest

from test_backend import Kind, Req

pytestmark = pytest.mark.gpu


def test_backend_end_to_end(cuda_ok):
    from m3_memory_b200.backend import M3Backend

    rng = np.random.default_rng(5)
    d, n = 24, 300
    C = rng.standard_normal((4, d)).astype(np.float32)
    X = (C[rng.integers(0, 4, n)] + 0.4 * rng.standard_normal((n, d))).astype(np.float32)
    keys = [f"doc-{i}" for i in range(n)]
    b = M3Backend()
    b.create_index(1, SimpleNamespace(dim=d, metric="l2", params={"centroids": C}))
    r = b.execute([Req(Kind.INSERT, 1, ext_ids=keys, vectors=X),
                   Req(Kind.SEARCH, 1, vectors=X[:50], k=1, request_id="a")])
    assert r.upserted == n
    assert [h[0].id for h in r.searches["a"]] == keys[:50]
    moved = (X[10] + 5.0).astype(np.float32)[None]
    r = b.execute([Req(Kind.DELETE_IDS, 1, ext_ids=keys[:5]),
                   Req(Kind.UPDATE, 1, ext_ids=[keys[10]], vectors=moved),
                   Req(Kind.SEARCH, 1, vectors=X[:5], k=3, request_id="b"),
                   Req(Kind.SEARCH, 1, vectors=moved, k=1, request_id="c")])
    assert (r.deleted, r.updated) == (5, 1)
    for hits in r.searches["b"]:
        assert not {h.id for h in hits} & set(keys[:5])
    assert r.searches["c"][0][0].id == keys[10] and r.searches["c"][0][0].score < 1e-3
    b.close()
