"""The asynchronous write path (queue + writer threads) against the reference
core's AsyncEngine driven with the same operations."""
import numpy as np
import pytest

from gpu_common import engine_from_golden
from helpers import compare_search, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


@pytest.fixture
def ref_ok(have_ref):
    if not have_ref:
        pytest.skip("reference core library not built")


def _pair(cabi, oracle_mod, g):
    O = oracle_mod
    e = cabi.Engine()
    e.start(2, 0)
    r = O.RefEngine()
    r.start(2, 0)
    C = g["C"]
    d = C.shape[1]
    e.create_ivf(1, d, int(g["metric"]), bool(g["normalized"]), C)
    r.create_ivf(1, d, int(g["metric"]), bool(g["normalized"]), C)
    return e, r


def test_insert_update_delete_sequence(cabi, oracle_mod, ref_ok):
    g = load_golden("ip_mixture")
    e, r = _pair(cabi, oracle_mod, g)
    rng = np.random.default_rng(5)
    off, vecs, ids = g["off"], g["lvecs"], g["lids"]
    L = len(off) - 1
    for c in range(L):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            for eng in (e, r):
                assert eng.enqueue_insert(1, c, ids[b:t], vecs[b:t])
    for eng in (e, r):
        eng.flush()
    Q = g["Q"]
    compare_search(e.search(1, Q, 10, 4), r.search(1, Q, 10, 4))
    # update: overwrite some rows, append new ids with insert_if_absent
    c = 3
    b, t = int(off[c]), int(off[c + 1])
    upd_ids = np.concatenate([ids[b:b + 5], np.array([900001, 900002])])
    upd_vecs = rng.standard_normal((7, vecs.shape[1])).astype(np.float32)
    for eng in (e, r):
        assert eng.enqueue_update(1, c, upd_ids, upd_vecs, True)
        assert eng.enqueue_delete(1, 5, ids[int(off[5]):int(off[5]) + 10])
        assert eng.enqueue_delete(1, 5, np.array([123456789]))  # absent: ignored
        eng.flush()
    compare_search(e.search(1, Q, 10, 6), r.search(1, Q, 10, 6))
    probe = upd_vecs[:3]
    compare_search(e.search(1, probe, 5, 8), r.search(1, probe, 5, 8))
    # compaction keeps results
    e.compact_cluster(1, 5)
    assert e.cluster_size(1, 5)[0] == e.cluster_size(1, 5)[1]
    compare_search(e.search(1, Q, 10, 6), r.search(1, Q, 10, 6))
    e.stop()
    r.stop()


def test_insert_auto_matches_reference(cabi, oracle_mod, ref_ok):
    g = load_golden("cosine_norm")
    e, r = _pair(cabi, oracle_mod, g)
    vecs, ids = g["lvecs"], g["lids"]
    perm = np.random.default_rng(1).permutation(len(ids))
    for s in range(0, len(perm), 400):
        sl = perm[s:s + 400]
        for eng in (e, r):
            assert eng.enqueue_insert_auto(1, ids[sl], vecs[sl])
    for eng in (e, r):
        eng.flush()
    L = len(g["C"])
    for c in range(L):
        assert e.cluster_size(1, c)[0] == int(g["off"][c + 1] - g["off"][c])
    compare_search(e.search(1, g["Q"], 10, 4), r.search(1, g["Q"], 10, 4))
    e.stop()
    r.stop()


def test_writer_error_surfaces_at_flush(cabi):
    """A duplicate id kills the reference's writer thread (std::terminate); here
    the error is kept and raised by the next flush()."""
    e = cabi.Engine()
    e.start(1, 0)
    e.create_ivf(0, 8, cabi.L2, False, np.zeros((2, 8), np.float32))
    v = np.ones((3, 8), np.float32)
    assert e.enqueue_insert(0, 1, np.array([1, 2, 3]), v)
    e.flush()
    assert e.enqueue_insert(0, 1, np.array([3, 4, 5]), v)  # 3 exists
    with pytest.raises(cabi.M3GError, match="duplicate id exists"):
        e.flush()
    assert e.cluster_size(0, 1) == (3, 3)
    assert e.enqueue_insert(0, 1, np.array([6, 6]), v[:2])  # duplicate inside the batch
    with pytest.raises(cabi.M3GError, match="duplicate id in batch"):
        e.flush()
    assert e.enqueue_update(0, 1, np.array([7]), v[:1], False)  # absent, no insert
    with pytest.raises(cabi.M3GError, match="id not found"):
        e.flush()
    assert e.enqueue_insert(0, 9, np.array([8]), v[:1])  # bad cluster: std::out_of_range
    with pytest.raises(IndexError, match="invalid cluster_id"):
        e.flush()
    e.stop()
    assert not e.enqueue_insert(0, 0, np.array([8]), v[:1])  # stopped


def test_queue_full_nonblocking(cabi):
    e = cabi.Engine()
    e.create_ivf(0, 4, cabi.L2, False, np.zeros((1, 4), np.float32))
    e.set_queue_policy(capacity=1, pop_batch_max=1, block_on_full=False)
    e.start(1, 0)
    ok = [e.enqueue_insert(0, 0, np.array([i]), np.ones((1, 4), np.float32)) for i in range(200)]
    e.flush()
    assert any(ok)
    assert e.cluster_size(0, 0)[0] == sum(ok)
    e.stop()


def test_maintenance_compacts(cabi):
    e = cabi.Engine()
    e.create_ivf(0, 4, cabi.L2, False, np.zeros((1, 4), np.float32))
    e.start(1, 0)
    e.enqueue_insert(0, 0, np.arange(10), np.random.default_rng(0).random((10, 4)).astype(np.float32))
    e.enqueue_delete(0, 0, np.arange(5))
    e.flush()
    assert e.cluster_size(0, 0) == (10, 5)
    e.maintenance_pass(0)
    assert e.cluster_size(0, 0) == (5, 5)
    ids, sc, cnt = e.search(0, np.zeros((1, 4), np.float32), 10, 1)
    assert sorted(ids[0, :cnt[0]].tolist()) == [5, 6, 7, 8, 9]
    e.stop()


def test_updates_and_deletes_addressed_to_every_list(cuda_ok, oracle_mod):
    """cluster_id -1: an update or delete applies to every list holding the id
    (an id stored in two lists is changed in both), ids held nowhere are ignored,
    and such an update cannot insert."""
    from m3_memory_b200 import cabi

    rng = np.random.default_rng(21)
    L, d, per = 5, 16, 40
    C = rng.standard_normal((L, d)).astype(np.float32)
    e = cabi.Engine()
    e.create_ivf(1, d, oracle_mod.IP, False, C)
    rows = {}
    for c in range(L):
        ids = np.arange(c * 1000, c * 1000 + per, dtype=np.int64)
        if c in (1, 3):
            ids[-1] = 999  # the same id in lists 1 and 3
        X = (C[c] + 0.3 * rng.standard_normal((per, d))).astype(np.float32)
        e.load_cluster(1, c, ids, X)
        rows[c] = (ids, X)
    e.start(1, 0)
    gone = np.array([5, 1007, 999, 4031, 123456], np.int64)  # 123456 is held nowhere
    assert e.enqueue_delete(1, -1, gone)
    new = np.array([2003, 3004], np.int64)
    nv = rng.standard_normal((2, d)).astype(np.float32)
    assert e.enqueue_update(1, -1, new, nv)
    e.flush()
    with pytest.raises(ValueError):
        e.enqueue_update(1, -1, new, nv, insert_if_absent=True)
    for c in range(L):
        ids, X = rows[c]
        keep = ~np.isin(ids, gone)
        want_ids, want_X = ids[keep], X[keep].copy()
        for i, v in zip(new, nv):
            want_X[want_ids == i] = v
        got_ids, got_X = e.get_cluster(1, c)
        np.testing.assert_array_equal(got_ids, want_ids)
        np.testing.assert_array_equal(got_X, want_X)
    e.stop()
