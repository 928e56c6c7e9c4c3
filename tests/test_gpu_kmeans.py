"""k-means and split on the GPU against the oracle restatement, bit-exact:
the E-step is the reference's nearest_clusters rule, the M-step is the fp64
ascending-row-order mean; both are deterministic."""
import numpy as np
import pytest

from helpers import KMEANS_CASES, compare_search, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


@pytest.mark.parametrize("case", KMEANS_CASES)
def test_kmeans_bit_exact(cabi, case):
    g = load_golden(case)
    e = cabi.Engine()
    C, a = e.kmeans(g["X"], int(g["nlist"]), int(g["niter"]), int(g["seed"]), int(g["metric"]),
                    bool(g["normalized"]))
    np.testing.assert_array_equal(a, g["assign"])
    np.testing.assert_array_equal(C, g["C"])


@pytest.mark.parametrize("case", KMEANS_CASES)
def test_split_bit_exact(cabi, case):
    g = load_golden(case)
    X, assign, C = g["X"], g["assign"], g["C"]
    nlist, d = C.shape
    e = cabi.Engine()
    e.create_ivf(4, d, int(g["metric"]), bool(g["normalized"]), C)
    rows = np.nonzero(assign == 0)[0]
    e.load_cluster(4, 0, rows.astype(np.int64) + 1000, X[rows])
    nid = e.split_cluster(4, 0, 5, int(g["split_seed"]))
    assert nid == nlist and e.info(4)[3] == nlist + 1
    Cg = e.centroids(4)
    np.testing.assert_array_equal(Cg[0], g["split_C"][0])
    np.testing.assert_array_equal(Cg[nlist], g["split_C"][1])
    sa = g["split_assign"]
    assert e.cluster_size(4, 0) == (int((sa == 0).sum()),) * 2
    assert e.cluster_size(4, nlist) == (int((sa == 1).sum()),) * 2
    # the moved rows are searchable in their new list, in list order
    ids, sc, cnt = e.search_on(4, np.array([nlist], np.int32), X[rows[sa == 1][:3]], 1)
    np.testing.assert_array_equal(ids[:, 0], rows[sa == 1][:3] + 1000)


def test_split_too_small(cabi):
    e = cabi.Engine()
    e.create_ivf(0, 8, cabi.L2, False, np.zeros((2, 8), np.float32))
    e.load_cluster(0, 1, np.array([5]), np.ones((1, 8), np.float32))
    assert e.split_cluster(0, 1) == -1
    assert e.split_cluster(0, 0) == -1


def test_train_ivf_then_search(cabi, oracle_mod):
    O = oracle_mod
    g = load_golden("kmeans_ip")
    X = g["X"]
    ids = np.arange(len(X), dtype=np.int64) * 3
    e = cabi.Engine()
    C = e.train_ivf(2, X.shape[1], int(g["metric"]), False, ids, X, int(g["nlist"]),
                    int(g["niter"]), int(g["seed"]))
    np.testing.assert_array_equal(C, g["C"])
    lists = O.CsrLists.from_assign(X, ids, g["assign"], int(g["nlist"]))
    Q = X[::37] + 0.01
    compare_search(e.search(2, Q, 10, 3), O.search_nprobe(Q, C, lists, int(g["metric"]), False, 10, 3))
