"""The tensor-core list scan (the default for every metric with k <= 128)
against the oracle, and against the SIMT scan (M3G_SCAN=simt, run in a child
process because the choice is read once per process).

The cases exercise the scan's structure: a list longer than one pass of row
blocks (2100 rows), ragged last blocks, dimensions that are not a multiple of
32 or 64, empty and tiny lists, erased rows, items of up to 32 queries (k <= 32)
or 16 queries (k <= 128, four register entries per lane), k up to 128, squared
L2 (ranked by its expansion, rescored exactly at the merge) and both cosine
forms."""
import os
import subprocess
import sys
import zlib
from pathlib import Path

import numpy as np
import pytest

from helpers import compare_search

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

SIZES = [0, 5, 130, 300, 1200, 2100, 1]
# name: metric, normalized, dim, nq, nprobe, k  (metric: 0 L2, 1 IP, 2 COSINE)
CASES = {
    "ip_wide_items": (1, False, 96, 40, 2, 10),     # 80 pairs over 7 lists
    "ip_narrow_items": (1, False, 96, 40, 1, 10),   # one probe: tiny lists alone
    "cos_raw_k32": (2, False, 64, 48, 3, 32),
    "cos_norm_all": (2, True, 128, 30, -1, 7),
    "l2_k10": (0, False, 96, 40, 2, 10),
    "l2_k100_dim100": (0, False, 100, 40, 3, 100),
    "ip_k64": (1, False, 96, 40, 3, 64),
    "cos_raw_k128": (2, False, 64, 24, 4, 128),
    "l2_k33_all": (0, False, 36, 20, -1, 33),
}


def make_case(name):
    metric, normalized, d, nq, nprobe, k = CASES[name]
    rng = np.random.default_rng(zlib.crc32(name.encode()))  # same data in the child process
    L = len(SIZES)
    C = rng.standard_normal((L, d)).astype(np.float32)
    n = sum(SIZES)
    owner = np.repeat(np.arange(L), SIZES)
    X = (C[owner] + 0.7 * rng.standard_normal((n, d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.7 * rng.standard_normal((nq, d))).astype(np.float32)
    if normalized:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
        C /= np.linalg.norm(C, axis=1, keepdims=True)
    ids = (np.arange(n, dtype=np.int64) * 7 + 3)
    alive = np.ones(n, np.uint8)
    alive[rng.random(n) < 0.05] = 0  # erased rows
    off = np.concatenate([[0], np.cumsum(SIZES)]).astype(np.int64)
    return dict(metric=metric, normalized=normalized, C=C, X=X, Q=Q, ids=ids, alive=alive,
                off=off, nprobe=nprobe, k=k)


def engine_search(cabi, case):
    e = cabi.Engine()
    d = case["C"].shape[1]
    e.create_ivf(1, d, case["metric"], case["normalized"], case["C"])
    off, ids, X, alive = case["off"], case["ids"], case["X"], case["alive"]
    for c in range(len(off) - 1):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            e.load_cluster(1, c, ids[b:t], X[b:t])
    e.start(1, 0)
    for c in range(len(off) - 1):
        b, t = int(off[c]), int(off[c + 1])
        dead = ids[b:t][alive[b:t] == 0]
        if len(dead):
            assert e.enqueue_delete(1, c, dead)
    e.flush()
    out = e.search(1, case["Q"], case["k"], case["nprobe"])
    e.stop()
    return out


CHILD = r'''
import sys, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from m3_memory_b200 import cabi
import test_gpu_scan_paths as T
out = {}
for name in T.CASES:
    ids, sc, cnt = T.engine_search(cabi, T.make_case(name))
    out[name + "_ids"], out[name + "_sc"], out[name + "_cnt"] = ids, sc, cnt
np.savez(sys.argv[2], **out)
'''


@pytest.mark.parametrize("name", list(CASES))
def test_tensor_core_scan_matches_oracle(cuda_ok, oracle_mod, name):
    from m3_memory_b200 import cabi

    case = make_case(name)
    got = engine_search(cabi, case)
    lists = oracle_mod.CsrLists(case["off"], case["X"], case["ids"], case["alive"])
    ref = oracle_mod.search_nprobe(case["Q"], case["C"], lists, case["metric"],
                                   case["normalized"], case["k"], case["nprobe"])
    compare_search(got, ref)


def test_tensor_core_and_simt_scans_agree(cuda_ok, tmp_path):
    from m3_memory_b200 import cabi

    f = tmp_path / "simt.npz"
    env = dict(os.environ, M3G_SCAN="simt")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(f)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    simt = np.load(f)
    for name in CASES:
        got = engine_search(cabi, make_case(name))
        ref = (simt[name + "_ids"], simt[name + "_sc"], simt[name + "_cnt"])
        # both are fp32-accurate restatements: same counts, near-identical scores
        compare_search(got, ref, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("metric", [0, 1, 2])
def test_exact_duplicates_across_lists_keep_the_reference_order(cuda_ok, oracle_mod, metric):
    """The same 24 vectors stored in each of 6 lists (plus distinct rows): the
    top-k is made of exact score ties across lists.  Rows tying the per-query
    bound of the tensor-core scan (a finished list's k-th score) must stay in:
    the exact scores of the rows returned must be the oracle's, position by
    position (which copies fill a tie group at the k-th place is left open, as
    the reference's final sort leaves it)."""
    from m3_memory_b200 import cabi

    rng = np.random.default_rng(77 + metric)
    d, L, nq = 64, 6, 16
    C = rng.standard_normal((L, d)).astype(np.float32)
    base = rng.standard_normal((24, d)).astype(np.float32)
    rows, lid = [], []
    for c in range(L):
        rows += [base, (C[c] + 0.3 * rng.standard_normal((40 + 7 * c, d))).astype(np.float32)]
        lid += [c] * (24 + 40 + 7 * c)
    X = np.concatenate(rows)
    sizes = np.bincount(lid, minlength=L)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    ids = np.arange(len(X), dtype=np.int64) * 5 + 2
    Q = (base[rng.integers(0, 24, nq)] + 0.05 * rng.standard_normal((nq, d))).astype(np.float32)
    case = dict(metric=metric, normalized=False, C=C, X=X, Q=Q, ids=ids,
                alive=np.ones(len(X), np.uint8), off=off, nprobe=5, k=10)
    got = engine_search(cabi, case)
    lists = oracle_mod.CsrLists(off, X, ids, case["alive"])
    ref = oracle_mod.search_nprobe(Q, C, lists, metric, False, 10, 5)
    np.testing.assert_array_equal(got[2], ref[2])
    row_of = {int(i): r for r, i in enumerate(ids)}
    for q in range(nq):
        c = int(ref[2][q])
        exact = [oracle_mod.score(Q[q], X[row_of[int(i)]], metric, False) for i in got[0][q, :c]]
        np.testing.assert_array_equal(np.array(exact, np.float32), ref[1][q, :c], err_msg=str(q))
    compare_search(got, ref)


@pytest.mark.parametrize("k", [10, 100])
def test_l2_queries_on_stored_rows_get_exact_scores(cuda_ok, oracle_mod, k):
    """Queries equal to stored rows (distance 0) and a hair away from them: the
    expansion ||x||^2 - 2<x,q> + ||q||^2 cannot resolve these, the merge's exact
    rescoring must -- every returned score is the reference's own sum of
    squared differences, and the stored row itself comes first."""
    from m3_memory_b200 import cabi

    rng = np.random.default_rng(5 + k)
    d, L = 192, 8
    C = (3.0 * rng.standard_normal((L, d))).astype(np.float32)
    sizes = [300, 520, 10, 0, 410, 130, 999, 64]
    owner = np.repeat(np.arange(L), sizes)
    X = (C[owner] + rng.standard_normal((len(owner), d))).astype(np.float32)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    pick = rng.choice(len(X), 24, replace=False)
    Q = X[pick].copy()
    Q[12:] += np.float32(1e-3) * rng.standard_normal((12, d)).astype(np.float32)
    ids = np.arange(len(X), dtype=np.int64) + 1000
    case = dict(metric=0, normalized=False, C=C, X=X, Q=Q, ids=ids,
                alive=np.ones(len(X), np.uint8), off=off, nprobe=3, k=k)
    got = engine_search(cabi, case)
    lists = oracle_mod.CsrLists(off, X, ids, case["alive"])
    ref = oracle_mod.search_nprobe(Q, C, lists, 0, False, k, 3)
    np.testing.assert_array_equal(got[2], ref[2])
    for q in range(len(Q)):
        c = int(ref[2][q])
        exact = [oracle_mod.score(Q[q], X[int(i) - 1000], 0, False) for i in got[0][q, :c]]
        np.testing.assert_array_equal(np.array(exact, np.float32), got[1][q, :c], err_msg=str(q))
        if q < 12:
            assert got[0][q, 0] == ids[pick[q]] and got[1][q, 0] == 0.0
    compare_search(got, ref)
