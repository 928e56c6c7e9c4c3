"""The online insert + split stream: batches of rows routed by
enqueue_insert_auto (AgentMemory/M3/src/m3_async.cpp:262-313), then one split
pass that splits every list over twice the mean size by 2-means (5 rounds), then
searches.  The reference has no split (its TODO, AgentMemory/M3/src/
m3_index.cpp:304-311), so the oracle replays the same pass into the reference
core with the primitives the TODO names (set_centroid, add_cluster,
rebuild_cluster, :133-163) and routes the inserts with the reference's own
nearest_clusters and add_batch.  After every batch the centroids must be
bit-identical and the searches must match the reference core's."""
import numpy as np
import pytest

from helpers import compare_search

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric,normalized", [(1, False), (0, False)])
def test_insert_split_stream_matches_reference(cuda_ok, oracle_mod, have_ref, metric, normalized):
    if not have_ref:
        pytest.skip("the reference core (oracle/_ref/liboracle_ref.so) is not built")
    O = oracle_mod
    from m3_memory_b200 import cabi, synthetic as S

    rng = np.random.default_rng(21 + metric)
    d, L, n0 = 96, 48, 12000
    means = S.mixture_means(40, d, rng)
    X0, _ = S.gaussian_mixture(n0, means, 0.3, rng)
    e = cabi.Engine()
    ids0 = np.arange(n0, dtype=np.int64)
    C = e.train_ivf(1, d, metric, normalized, ids0, X0, L, 4, 3)
    a0 = e.nearest_clusters(1, X0)
    ref = O.RefIndex(d, metric, normalized)
    ref.set_centroids(C)
    rows = []
    for c in range(L):
        sel = np.flatnonzero(a0 == c)
        rows.append((ids0[sel], X0[sel]))
        if len(sel):
            ref.rebuild_cluster(c, ids0[sel], X0[sel])
    e.start(2, 0)
    shifted = S.shifted_means(means, 0.5, rng)
    next_id = n0
    splits = 0
    for batch in range(6):
        Xb, _ = S.gaussian_mixture(1500, shifted[:8], 0.3, rng)  # a few regions grow
        ib = np.arange(next_id, next_id + len(Xb), dtype=np.int64)
        next_id += len(Xb)
        assert e.enqueue_insert_auto(1, ib, Xb)
        e.flush()
        # the reference: its own routing, then add_batch per cluster (row order kept)
        route = ref.nearest_clusters(Xb)
        for c in np.unique(route):
            sel = np.flatnonzero(route == c)
            ref.add_batch(int(c), ib[sel], Xb[sel])
            rows[c] = (np.concatenate([rows[c][0], ib[sel]]), np.concatenate([rows[c][1], Xb[sel]]))
        got_new = e.split_oversized(1, 2.0, 5, 100)
        want_new = O.split_oversized(ref, rows, 2.0, 5, 100, metric, normalized)
        assert got_new == len(want_new)
        splits += got_new
        Cg = e.centroids(1)
        assert Cg.shape[0] == len(rows)
        for c in range(len(rows)):
            size, live = e.cluster_size(1, c)
            assert live == len(rows[c][0]), (batch, c)
        Q, _ = S.gaussian_mixture(64, shifted, 0.3, rng)
        got = e.search(1, Q, 10, 6)
        want = ref.search_nprobe(Q, 10, 6)
        compare_search(got, want)
    e.stop()
    assert splits > 0
    # the final centroids: the reference's after the same splits
    for c in range(len(rows)):
        gi, gv = e.get_cluster(1, c)
        np.testing.assert_array_equal(np.sort(gi), np.sort(rows[c][0]))
