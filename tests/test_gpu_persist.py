"""Native save / load of an index and the read-back of a list's live rows.

An index built from each golden case (erased rows included) is saved, loaded
into a second engine, and must answer every search exactly as the original;
the lists read back must hold the case's live rows, bit for bit; a damaged
file must leave the target index as it was."""
import numpy as np
import pytest

from gpu_common import engine_from_golden
from helpers import INDEX_CASES, lists_of, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


@pytest.mark.parametrize("case", INDEX_CASES)
def test_save_load_round_trip(cabi, case, tmp_path):
    g = load_golden(case)
    e = engine_from_golden(cabi, g)
    off, vecs, ids, alive = lists_of(g)
    L = len(off) - 1
    for c in range(L):
        b, t = int(off[c]), int(off[c + 1])
        keep = alive[b:t] != 0
        got_ids, got_vecs = e.get_cluster(1, c)
        np.testing.assert_array_equal(got_ids, ids[b:t][keep])
        np.testing.assert_array_equal(got_vecs, vecs[b:t][keep])
    path = tmp_path / "index.m3g"
    e.save_index(1, path)
    e2 = cabi.Engine()
    e2.load_index(7, path)
    assert e2.info(7) == e.info(1)
    np.testing.assert_array_equal(e2.centroids(7), e.centroids(1))
    for c in range(L):
        a_ids, a_vecs = e.get_cluster(1, c)
        b_ids, b_vecs = e2.get_cluster(7, c)
        np.testing.assert_array_equal(a_ids, b_ids)
        np.testing.assert_array_equal(a_vecs, b_vecs)
    k = int(g["k"])
    for p in g["nprobes"].tolist():
        p = p if p > 0 else L
        want = e.search(1, g["Q"], k, p)
        got = e2.search(7, g["Q"], k, p)
        for w, x in zip(want, got):
            np.testing.assert_array_equal(x, w)


def test_damaged_file_changes_nothing(cabi, tmp_path):
    g = load_golden("ip_mixture")
    e = engine_from_golden(cabi, g)
    path = tmp_path / "index.m3g"
    e.save_index(1, path)
    data = path.read_bytes()
    want = e.search(1, g["Q"], 5, 3)
    (tmp_path / "short.m3g").write_bytes(data[: len(data) // 2])
    with pytest.raises(RuntimeError):
        e.load_index(1, tmp_path / "short.m3g")
    (tmp_path / "foreign.m3g").write_bytes(b"NOTANIDX" + data[8:])
    with pytest.raises(ValueError):
        e.load_index(1, tmp_path / "foreign.m3g")
    with pytest.raises(RuntimeError):
        e.load_index(1, tmp_path / "missing.m3g")
    for w, x in zip(want, e.search(1, g["Q"], 5, 3)):
        np.testing.assert_array_equal(x, w)


def test_pybind_save_load(cuda_ok, tmp_path):
    from m3_memory_b200 import _m3_async as m3

    rng = np.random.default_rng(3)
    C = rng.standard_normal((6, 32)).astype(np.float32)
    X = (C[rng.integers(0, 6, 500)] + 0.3 * rng.standard_normal((500, 32))).astype(np.float32)
    eng = m3.AsyncEngine()
    eng.start()
    eng.create_ivf(2, 32, m3.Metric.IP, False, C)
    assert eng.enqueue_insert_auto(2, np.arange(500, dtype=np.int64), X)
    eng.flush()
    path = str(tmp_path / "pb.m3g")
    eng.save_index(2, path)
    other = m3.AsyncEngine()
    other.load_index(4, path)
    Q = X[:20]
    assert other.search(4, Q, 5, 3) == eng.search(2, Q, 5, 3)
    eng.stop()
