"""Faiss IndexIVFFlat import (rebuild_from_faiss, AgentMemory/M3/faiss_loader.py:
24-79) read by the engine itself.  The files come from tests/faiss_format.py,
written from Faiss's published layout (faiss is not installed, so parity with
real Faiss files is unpinned); the imported index must hold exactly the lists
and centroids written and answer as the oracle does over them."""
import numpy as np
import pytest

from faiss_format import FAISS_IP, FAISS_L2, write_ivfflat
from helpers import compare_search

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


def make(rng, L, d, sizes):
    C = rng.standard_normal((L, d)).astype(np.float32)
    lists, base = [], 0
    for c, n in enumerate(sizes):
        ids = (np.arange(n, dtype=np.int64) + base) * 13 + 7
        base += n
        lists.append((ids, (C[c] + 0.5 * rng.standard_normal((n, d))).astype(np.float32)))
    return C, lists


@pytest.mark.parametrize("fmetric,sparse,direct_map", [(FAISS_L2, False, 0), (FAISS_IP, True, 1),
                                                       (FAISS_L2, True, 2)])
def test_faiss_ivfflat_import(cabi, oracle_mod, tmp_path, fmetric, sparse, direct_map):
    O = oracle_mod
    rng = np.random.default_rng(fmetric * 10 + direct_map)
    d = 48
    sizes = [0, 40, 0, 0, 300, 9, 0, 120] if sparse else [50, 0, 200, 31, 77]
    C, lists = make(rng, len(sizes), d, sizes)
    path = tmp_path / "ivf.faiss"
    write_ivfflat(path, C, lists, fmetric, sparse, direct_map)
    from m3_memory_b200.faiss_loader import rebuild_from_faiss

    e = cabi.Engine()
    rebuild_from_faiss(e, index_id=3, path=path, normalized=False)
    dim, metric, norm, L = e.info(3)
    assert (dim, L, norm) == (d, len(sizes), False)
    assert metric == (cabi.L2 if fmetric == FAISS_L2 else cabi.IP)
    np.testing.assert_array_equal(e.centroids(3), C)
    for c, (ids, vecs) in enumerate(lists):
        gi, gv = e.get_cluster(3, c)
        np.testing.assert_array_equal(gi, ids)
        np.testing.assert_array_equal(gv, vecs)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    allv = np.concatenate([v for _, v in lists])
    alli = np.concatenate([i for i, _ in lists])
    Q = (C[rng.integers(0, len(sizes), 20)] + 0.5 * rng.standard_normal((20, d))).astype(np.float32)
    m = cabi.L2 if fmetric == FAISS_L2 else cabi.IP
    compare_search(e.search(3, Q, 10, 3),
                   O.search_nprobe(Q, C, O.CsrLists(off, allv, alli), m, False, 10, 3))


def test_faiss_import_refuses_damaged_files(cabi, tmp_path):
    rng = np.random.default_rng(1)
    C, lists = make(rng, 3, 16, [5, 6, 7])
    good = tmp_path / "good.faiss"
    n = write_ivfflat(good, C, lists)
    e = cabi.Engine()
    e.create_ivf(1, 16, cabi.L2, False, C)
    e.load_cluster(1, 0, np.array([1, 2]), np.ones((2, 16), np.float32))
    raw = good.read_bytes()
    bad = tmp_path / "bad.faiss"
    for blob, err in [(raw[: n - 9], RuntimeError),          # truncated in the last list
                      (b"IwPQ" + raw[4:], cabi.M3GError),      # another index type
                      (raw[:4] + b"\x00\x00\x00\x00" + raw[8:], ValueError)]:  # d = 0
        bad.write_bytes(blob)
        with pytest.raises(err):
            e.rebuild_from_faiss(1, bad)
        # a refused file leaves the index as it was
        assert e.info(1)[3] == 3 and e.cluster_size(1, 0) == (2, 2)
    with pytest.raises((RuntimeError, FileNotFoundError)):
        e.rebuild_from_faiss(1, tmp_path / "missing.faiss")
    # another quantizer type is refused too
    write_ivfflat(bad, C, lists, quantizer_tag=b"IxHE")
    with pytest.raises(cabi.M3GError) as ei:
        e.rebuild_from_faiss(1, bad)
    assert ei.value.code == cabi.M3G_EUNSUPPORTED


def test_backend_rebuild_then_update_and_delete(cuda_ok, tmp_path):
    """M3Backend.rebuild_index_from_faiss (AgentMemory/backend/m3.py:188-198): the
    imported ids are known to the backend, so an UPDATE of one replaces it in its
    list and a DELETE_IDS removes it."""
    from m3_memory_b200.backend import M3Backend

    rng = np.random.default_rng(4)
    C, lists = make(rng, 4, 32, [20, 30, 0, 25])
    path = tmp_path / "b.faiss"
    write_ivfflat(path, C, lists, FAISS_L2)
    be = M3Backend(default_nprobe=4)

    class Req:
        def __init__(self, op, **kw):
            self.op = op
            self.index_id = 0
            self.__dict__.update(kw)

    be.rebuild_index_from_faiss(0, path=str(path), normalized=False)
    target_id, target_vec = int(lists[1][0][3]), lists[1][1][3]
    far = (target_vec + 50.0).astype(np.float32)
    be.execute([Req("UPDATE", ext_ids=[target_id], vectors=far[None])])
    r = be.execute([Req("SEARCH", vectors=far[None], k=1, request_id="q")])
    assert r.searches["q"][0][0].id == str(target_id)
    assert r.searches["q"][0][0].score == pytest.approx(0.0, abs=1e-3)
    be.execute([Req("DELETE_IDS", ext_ids=[target_id])])
    r = be.execute([Req("SEARCH", vectors=far[None], k=5, request_id="q")])
    assert str(target_id) not in [h.id for h in r.searches["q"][0]]
    be.close()
