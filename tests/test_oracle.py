"""The oracle, pinned: the C restatement against the golden vectors the
reference core produced, and against the reference core itself when its
library is built (oracle/_ref/liboracle_ref.so)."""
import numpy as np
import pytest

from helpers import INDEX_CASES, KMEANS_CASES, compare_search, load_golden, lists_of


@pytest.mark.parametrize("case", INDEX_CASES)
def test_restatement_matches_golden_search(oracle_mod, case):
    O = oracle_mod
    g = load_golden(case)
    off, vecs, ids, alive = lists_of(g)
    lists = O.CsrLists(off, vecs, ids, alive)
    for p in g["nprobes"].tolist():
        got = O.search_nprobe(g["Q"], g["C"], lists, int(g["metric"]), bool(g["normalized"]),
                              int(g["k"]), p)
        ref = (g[f"ref_ids_p{p}"], g[f"ref_scores_p{p}"], g[f"ref_counts_p{p}"])
        compare_search(got, ref, exact=True)


@pytest.mark.parametrize("case", INDEX_CASES)
def test_restatement_matches_golden_assignment(oracle_mod, case):
    O = oracle_mod
    g = load_golden(case)
    # rows back in CSR order with their assignment = the list they sit in
    off = g["off"]
    want = np.repeat(np.arange(len(off) - 1, dtype=np.int32), np.diff(off))
    got = O.nearest_clusters(g["lvecs"], g["C"], int(g["metric"]), bool(g["normalized"]))
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("case", KMEANS_CASES)
def test_restatement_kmeans_is_pinned(oracle_mod, case):
    O = oracle_mod
    g = load_golden(case)
    C, a = O.kmeans_train(g["X"], int(g["nlist"]), int(g["niter"]), int(g["seed"]),
                          int(g["metric"]), bool(g["normalized"]))
    np.testing.assert_array_equal(C, g["C"])
    np.testing.assert_array_equal(a, g["assign"])
    C2, a2 = O.split_2means(g["X"][g["assign"] == 0], 5, int(g["split_seed"]), int(g["metric"]),
                            bool(g["normalized"]))
    np.testing.assert_array_equal(C2, g["split_C"])
    np.testing.assert_array_equal(a2, g["split_assign"])


def test_sampler_distinct_and_seeded(oracle_mod):
    O = oracle_mod
    s = O.sample_rows(5, 1000, 300)
    assert len(set(s.tolist())) == 300 and s.min() >= 0 and s.max() < 1000
    np.testing.assert_array_equal(s, O.sample_rows(5, 1000, 300))
    assert not np.array_equal(s, O.sample_rows(6, 1000, 300))
    with pytest.raises(ValueError):
        O.sample_rows(1, 3, 4)


def test_planted_mistake_is_caught(oracle_mod):
    """The checker must notice a wrong score or a wrong id."""
    O = oracle_mod
    g = load_golden("ip_mixture")
    lists = O.CsrLists(*lists_of(g))
    ids, sc, cnt = O.search_nprobe(g["Q"], g["C"], lists, int(g["metric"]), False, 10, 3)
    ref = (g["ref_ids_p3"], g["ref_scores_p3"], g["ref_counts_p3"])
    bad = sc.copy()
    bad[0, 0] += 1e-2
    with pytest.raises(AssertionError):
        compare_search((ids, bad, cnt), ref)
    bad_ids = ids.copy()
    bad_ids[:, 0] = -5  # every query loses a true neighbour: recall 0.9
    with pytest.raises(AssertionError):
        compare_search((bad_ids, sc, cnt), ref)


# ---- against the live reference core (built here from the reference sources) ----

def _random_index(O, metric, normalized, n, d, nlist, seed):
    from m3_memory_b200 import synthetic as S

    rng = np.random.default_rng(seed)
    X = S.unit_gaussian(n, d, rng)
    if not normalized and metric != O.IP:
        X = X * rng.uniform(0.3, 2.5, (n, 1)).astype(np.float32)
    X = np.ascontiguousarray(X, np.float32)
    Q = S.unit_gaussian(25, d, rng)
    C, a = O.kmeans_train(X, nlist, 3, seed, metric, normalized)
    return X, Q, C, a


@pytest.mark.parametrize("metric,normalized", [(0, False), (1, False), (2, True), (2, False)])
def test_restatement_matches_reference_core(oracle_mod, have_ref, metric, normalized):
    if not have_ref:
        pytest.skip("reference core library not built (no reference tree on this box)")
    O = oracle_mod
    X, Q, C, a = _random_index(O, metric, normalized, 2500, 48, 20, 100 + metric)
    ref = O.RefIndex(48, metric, normalized)
    ref.set_centroids(C)
    np.testing.assert_array_equal(ref.nearest_clusters(X), a)
    lists = O.CsrLists.from_assign(X, np.arange(len(X)) * 5 + 1, a, 20)
    lists.to_ref(ref)
    for k, p in [(10, 4), (1, 1), (40, 0), (5, 99)]:
        compare_search(O.search_nprobe(Q, C, lists, metric, normalized, k, p),
                       ref.search_nprobe(Q, k, p), exact=True)
    # search_on with an explicit (unsorted, partly out-of-range) cluster list
    cids = np.array([7, 3, -1, 25, 11], np.int32)
    compare_search(O.search_on(Q, lists, cids, metric, normalized, 10), ref.search_on(cids, Q, 10),
                   exact=True)


def test_engine_default_nprobe(oracle_mod, have_ref):
    """AsyncEngine::search maps nprobe <= 0 to default_nprobe (m3_async.cpp:224)."""
    if not have_ref:
        pytest.skip("reference core library not built")
    O = oracle_mod
    X, Q, C, a = _random_index(O, O.L2, False, 1500, 32, 16, 7)
    eng = O.RefEngine()
    eng.create_ivf(1, 32, O.L2, False, C)
    lists = O.CsrLists.from_assign(X, np.arange(len(X)), a, 16)
    for c in range(16):
        i, v = lists.rows(c)
        if len(i):
            eng.load_cluster(1, c, i, v)
    for dn in (8, 3):
        eng.set_search_policy(dn)
        compare_search(eng.search(1, Q, 10, 0),
                       O.search_nprobe(Q, C, lists, O.L2, False, 10, dn), exact=True)


@pytest.mark.parametrize("metric,normalized", [(1, False), (2, True), (0, False)])
def test_fast_assignment_equals_exact(oracle_mod, metric, normalized):
    """The BLAS-proposed, bound-filtered, exactly rescored assignment equals the
    plain nearest_clusters rule bit for bit, also with exact duplicate centroids
    (ties to the lower id) and near-duplicates inside the error bound."""
    O = oracle_mod
    rng = np.random.default_rng(40 + metric)
    d = 200
    means = rng.standard_normal((6, d)).astype(np.float32)
    X = (means[rng.integers(0, 6, 4000)] + 0.3 * rng.standard_normal((4000, d))).astype(np.float32)
    C = X[rng.choice(4000, 150, replace=False)].copy()
    C[60] = C[7]
    C[61] = np.nextafter(C[7], np.float32(np.inf))
    X[:20] = C[7]
    if normalized:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        C /= np.linalg.norm(C, axis=1, keepdims=True)
    stats = {}
    got = O.nearest_clusters_fast(X, C, metric, normalized, block=1024, stats=stats)
    np.testing.assert_array_equal(got, O.nearest_clusters(X, C, metric, normalized))
    assert stats["rescored_rows"] >= 20  # the rows sitting on the duplicated centroid


@pytest.mark.parametrize("case", KMEANS_CASES)
def test_fast_kmeans_equals_restatement(oracle_mod, case):
    O = oracle_mod
    g = load_golden(case)
    C, a = O.kmeans_train_fast(g["X"], int(g["nlist"]), int(g["niter"]), int(g["seed"]),
                               int(g["metric"]), bool(g["normalized"]))
    np.testing.assert_array_equal(C, g["C"])
    np.testing.assert_array_equal(a, g["assign"])
