"""Search parity on the GPU: the CUDA path (through the C ABI) against the
reference core's outputs (golden vectors) and the oracle restatement."""
import numpy as np
import pytest

from gpu_common import engine_from_golden, expected_probes
from helpers import INDEX_CASES, compare_search, load_golden, lists_of

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


@pytest.mark.parametrize("case", INDEX_CASES)
def test_search_matches_reference(cabi, case):
    g = load_golden(case)
    e = engine_from_golden(cabi, g)
    for p in g["nprobes"].tolist():
        got = e.search(1, g["Q"], int(g["k"]), p if p > 0 else len(g["C"]))
        ref = (g[f"ref_ids_p{p}"], g[f"ref_scores_p{p}"], g[f"ref_counts_p{p}"])
        compare_search(got, ref)


@pytest.mark.parametrize("case", INDEX_CASES)
def test_nprobe_selection_bit_exact(cabi, oracle_mod, case):
    O = oracle_mod
    g = load_golden(case)
    e = engine_from_golden(cabi, g)
    metric, norm = int(g["metric"]), bool(g["normalized"])
    for p in (1, 3, len(g["C"]) // 2):
        got = e.select_probes(1, g["Q"], p)
        want = expected_probes(O, g["Q"], g["C"], metric, norm, p)
        for q in range(len(g["Q"])):
            if not np.array_equal(got[q], want[q]):
                # allowed only where the exact scores tie
                s_got = [O.score(g["Q"][q], g["C"][c], metric, norm) for c in got[q]]
                s_want = [O.score(g["Q"][q], g["C"][c], metric, norm) for c in want[q]]
                assert s_got == s_want, (case, p, q, got[q], want[q])


@pytest.mark.parametrize("case", INDEX_CASES)
def test_assignment_bit_exact(cabi, case):
    g = load_golden(case)
    e = engine_from_golden(cabi, g)
    off = g["off"]
    want = np.repeat(np.arange(len(off) - 1, dtype=np.int32), np.diff(off))
    np.testing.assert_array_equal(e.nearest_clusters(1, g["lvecs"]), want)


def test_search_on_matches_oracle(cabi, oracle_mod):
    O = oracle_mod
    g = load_golden("ip_mixture")
    e = engine_from_golden(cabi, g)
    lists = O.CsrLists(*lists_of(g))
    cids = np.array([5, 2, -4, 999, 17, 2 + 1], np.int32)
    got = e.search_on(1, cids, g["Q"], 10)
    ref = O.search_on(g["Q"], lists, cids, int(g["metric"]), False, 10)
    compare_search(got, ref)


def test_default_nprobe_and_clamping(cabi):
    g = load_golden("cosine_norm")
    e = engine_from_golden(cabi, g)
    L = len(g["C"])
    e.set_search_policy(default_nprobe=3)
    a = e.search(1, g["Q"], 10, 0)
    b = e.search(1, g["Q"], 10, 3)
    np.testing.assert_array_equal(a[0], b[0])
    # nprobe > nlist clamps to nlist (m3_index.cpp:388)
    c = e.search(1, g["Q"], 10, 10 * L)
    d = e.search(1, g["Q"], 10, L)
    np.testing.assert_array_equal(c[0], d[0])
    ref = (g["ref_ids_p32"], g["ref_scores_p32"], g["ref_counts_p32"])
    compare_search(c, ref)


def test_empty_and_unknown(cabi):
    e = cabi.Engine()
    Q = np.ones((3, 8), np.float32)
    ids, sc, cnt = e.search(7, Q, 5, 2)  # unknown index: empty (m3_async.cpp:218-222)
    assert (cnt == 0).all() and (ids == -1).all()
    e.create_ivf(2, 8, cabi.L2, False, np.zeros((0, 8), np.float32))
    ids, sc, cnt = e.search(2, Q, 5, 2)  # no lists
    assert (cnt == 0).all()
    e.create_ivf(3, 8, cabi.L2, False, np.eye(8, dtype=np.float32)[:4])
    ids, sc, cnt = e.search(3, Q, 5, 2)  # lists exist but are empty
    assert (cnt == 0).all()
    ids, sc, cnt = e.search(3, Q, 0, 2)  # k = 0
    assert (cnt == 0).all()
    assert (e.nearest_clusters(2, Q) == -1).all()


def test_k_above_limit_is_rejected(cabi):
    g = load_golden("cosine_norm")
    e = engine_from_golden(cabi, g)
    with pytest.raises(cabi.M3GError) as ei:
        e.search(1, g["Q"], 100000, 4)
    assert ei.value.code == cabi.M3G_EUNSUPPORTED


def test_odd_dimension_and_small_k(cabi, oracle_mod):
    """dim not a multiple of 4 (rows are zero padded on the device), k = 1."""
    O = oracle_mod
    rng = np.random.default_rng(3)
    X = rng.standard_normal((700, 37)).astype(np.float32)
    Q = rng.standard_normal((20, 37)).astype(np.float32)
    C, a = O.kmeans_train(X, 9, 3, 1, O.L2, False)
    lists = O.CsrLists.from_assign(X, np.arange(700) + 10, a, 9)
    e = cabi.Engine()
    e.create_ivf(0, 37, O.L2, False, C)
    for c in range(9):
        i, v = lists.rows(c)
        if len(i):
            e.load_cluster(0, c, i, v)
    for k, p in [(1, 2), (5, 9)]:
        compare_search(e.search(0, Q, k, p), O.search_nprobe(Q, C, lists, O.L2, False, k, p))


def test_host_query_batches_match_device_queries(cabi, oracle_mod):
    """The host-buffer search (queries copied into the engine's workspace, results
    copied back) gives the device-query path's answers bit for bit, on
    consecutive calls and batch sizes that are not multiples of the tile sizes."""
    import torch

    rng = np.random.default_rng(11)
    L, d = 300, 128
    C = rng.standard_normal((L, d)).astype(np.float32)
    assign = rng.integers(0, L, 20000)
    X = (C[assign] + 0.5 * rng.standard_normal((20000, d))).astype(np.float32)
    e = cabi.Engine()
    e.create_ivf(1, d, oracle_mod.IP, False, C)
    for c in range(L):
        rows = np.flatnonzero(assign == c)
        if len(rows):
            e.load_cluster(1, c, rows.astype(np.int64), X[rows])
    for nq in (700, 512, 1031):
        Q = (C[rng.integers(0, L, nq)] + 0.5 * rng.standard_normal((nq, d))).astype(np.float32)
        got = e.search(1, Q, 10, 17)
        qd = torch.from_numpy(Q).cuda()
        ids = torch.empty((nq, 10), dtype=torch.int64, device="cuda")
        sc = torch.empty((nq, 10), dtype=torch.float32, device="cuda")
        cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
        e.search_device(1, qd.data_ptr(), nq, 10, 17, ids.data_ptr(), sc.data_ptr(), cnt.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got[2], cnt.cpu().numpy())
        np.testing.assert_array_equal(got[0], ids.cpu().numpy())
        np.testing.assert_array_equal(got[1], sc.cpu().numpy())


@pytest.mark.parametrize("L", [5000, 9000])
def test_many_lists_match_oracle(cabi, oracle_mod, L):
    """Thousands of small lists (the work list's planner then takes several lists
    per thread, within and beyond the count it keeps in registers)."""
    rng = np.random.default_rng(L)
    d, n, nq = 32, 30000, 64
    C = rng.standard_normal((L, d)).astype(np.float32)
    assign = rng.integers(0, L, n)
    X = (C[assign] + 0.3 * rng.standard_normal((n, d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    ids = np.arange(n, dtype=np.int64) * 3
    e = cabi.Engine()
    e.create_ivf(1, d, oracle_mod.IP, False, C)
    order = np.argsort(assign, kind="stable")
    bounds = np.searchsorted(assign[order], np.arange(L + 1))
    for c in range(L):
        rows = order[bounds[c]:bounds[c + 1]]
        if len(rows):
            e.load_cluster(1, c, ids[rows], X[rows])
    lists = oracle_mod.CsrLists.from_assign(X, ids, assign, L)
    compare_search(e.search(1, Q, 5, 16), oracle_mod.search_nprobe(Q, C, lists, oracle_mod.IP,
                                                                  False, 5, 16))


def test_graph_replay_matches_direct_launches(cabi, oracle_mod):
    """A search batch shape is captured once as a CUDA graph and replayed; the
    answers equal those of the directly launched kernels (the stage-timed path),
    also after the index's lists change between replays."""
    rng = np.random.default_rng(8)
    L, d = 64, 96
    C = rng.standard_normal((L, d)).astype(np.float32)
    assign = rng.integers(0, L, 6000)
    X = (C[assign] + 0.4 * rng.standard_normal((6000, d))).astype(np.float32)
    e = cabi.Engine()
    e.create_ivf(1, d, oracle_mod.IP, False, C)
    for c in range(L):
        rows = np.flatnonzero(assign == c)
        e.load_cluster(1, c, rows.astype(np.int64), X[rows])
    Q = (C[rng.integers(0, L, 300)] + 0.4 * rng.standard_normal((300, d))).astype(np.float32)

    def direct():
        e.set_profiling(True)
        try:
            return e.search(1, Q, 10, 8)
        finally:
            e.set_profiling(False)

    for step in range(2):
        want = direct()
        for _ in range(3):  # capture, then replays
            got = e.search(1, Q, 10, 8)
            for w, x in zip(want, got):
                np.testing.assert_array_equal(x, w)
        # change two lists' contents between replays
        for c in (3, 5):
            rows = np.flatnonzero(assign == c)[: 10 + step]
            e.load_cluster(1, c, rows.astype(np.int64) + 100000, X[rows] * 1.5)
