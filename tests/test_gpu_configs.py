"""Parity on the benchmark configurations themselves, not only on small fixtures.

* The CPU-runnable configuration in full: 100k x 1024 unit-norm N(0, 1) rows,
  COSINE (normalized), nlist 256 by k-means (10 iterations, seeded random
  init), nprobe 16, k 10, 1000 queries in one batch.  The GPU's centroids and
  assignment must equal the oracle's k-means bit for bit; every query's nprobe
  selection must equal the oracle's (exact ties aside), and every query's answer
  must match the reference core's own search_nprobe (IVFIndex::search_nprobe,
  AgentMemory/M3/src/m3_index.cpp:368-483) on the same index.
* The headline search's coarse step: nlist 4096, dim 1024, nprobe 32, 256
  queries of a 1000-component mixture against k-means centroids of that
  mixture (close scores, so the exact rescoring decides many probes): the
  selection must equal the oracle's select_nprobe
  (select_nprobe_for_query, m3_index.cpp:492-523) except at exact ties.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from helpers import compare_search

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


def _threads():
    return max(1, len(os.sched_getaffinity(0)))


def _selection_matches(O, Q, C, metric, norm, got, p):
    """got[q] equals the oracle's top-p of query q, except between exactly tied scores."""
    def one(q):
        want = O.select_nprobe(Q[q], C, metric, norm, p)
        if np.array_equal(got[q], want):
            return None
        s_got = [O.score(Q[q], C[c], metric, norm) for c in got[q]]
        s_want = [O.score(Q[q], C[c], metric, norm) for c in want]
        return None if s_got == s_want else (q, got[q], want)

    with ThreadPoolExecutor(_threads()) as ex:
        bad = [r for r in ex.map(one, range(len(Q))) if r is not None]
    assert not bad, bad[:3]


def test_config1_full(cabi, oracle_mod, have_ref):
    O = oracle_mod
    from m3_memory_b200 import synthetic as S

    rng = np.random.default_rng(0)
    X = S.unit_gaussian(100_000, 1024, rng)
    Q = S.unit_gaussian(1000, 1024, rng)
    ids = np.arange(100_000, dtype=np.int64)
    e = cabi.Engine()
    C = e.train_ivf(1, 1024, O.COSINE, True, ids, X, 256, 10, 0)
    a = e.nearest_clusters(1, X)
    C_o, a_o = O.kmeans_train_fast(X, 256, 10, 0, O.COSINE, True)
    np.testing.assert_array_equal(C, C_o)
    np.testing.assert_array_equal(a, a_o)

    got = e.search(1, Q, 10, 16)
    assert (got[2] == 10).all()
    _selection_matches(O, Q, C_o, O.COSINE, True, e.select_probes(1, Q, 16), 16)
    lists = O.CsrLists.from_assign(X, ids, a_o, 256)
    if have_ref:
        ref = O.RefIndex(1024, O.COSINE, True)
        ref.set_centroids(C_o)
        lists.to_ref(ref)
        want = ref.search_nprobe(Q, 10, 16, threads=_threads())
    else:
        want = O.search_nprobe(Q, C_o, lists, O.COSINE, True, 10, 16)
    compare_search(got, want)


def test_headline_select_shape(cabi, oracle_mod):
    O = oracle_mod
    from m3_memory_b200 import synthetic as S

    rng = np.random.default_rng(5)
    means = S.mixture_means(1000, 1024, rng)
    X, _ = S.gaussian_mixture(300_000, means, 0.3, rng)
    Q, _ = S.gaussian_mixture(256, means, 0.3, rng)
    e = cabi.Engine()
    C, _ = e.kmeans(X, 4096, 3, 1, O.IP, False)
    e.create_ivf(1, 1024, O.IP, False, C)
    got = e.select_probes(1, Q, 32)
    assert got.shape == (256, 32)
    _selection_matches(O, Q, C, O.IP, False, got, 32)
