"""Row tiles of long lists in the tensor-core scan (m3g_set_scan_tile_rows).

A list longer than the tile and probed by at most two query groups is scanned
as row tiles spread over the SMs, each with its own partial top-k per (query,
probe); the last tile of a pair to finish merges them by (score, row in the
list).  The answers must not depend on the tiling: tiles of 128 rows, the
automatic size and no tiles give identical arrays, which match the oracle (the
reference's algorithm) as every scan does.  The cases cover
ragged last tiles, erased rows, every metric, k up to 128 with one query per
item (the epilogue's row split), a batch of one, bf16-stored rows, and a list
whose tiles do not fit the tile region (scanned whole beside tiled lists)."""
import zlib

import numpy as np
import pytest

from helpers import compare_search

pytestmark = pytest.mark.gpu

SIZES = [0, 5, 130, 300, 1200, 2100, 1, 4500, 777, 128, 256]
# name: metric, normalized, dim, nq, nprobe, k  (metric: 0 L2, 1 IP, 2 COSINE)
CASES = {
    "ip_k10": (1, False, 96, 40, 3, 10),
    "l2_k100_few_queries": (0, False, 100, 6, 4, 100),
    "cos_raw_k32": (2, False, 64, 48, 4, 32),
    "cos_norm_all_k7": (2, True, 128, 30, -1, 7),
    "ip_one_query_k128": (1, False, 64, 1, 5, 128),
    "ip_two_groups": (1, False, 48, 64, -1, 16),  # 64 queries per list: two groups per tile
    "l2_k33": (0, False, 36, 20, 6, 33),
}


def make_case(name, sizes=SIZES):
    metric, normalized, d, nq, nprobe, k = CASES[name]
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    L = len(sizes)
    C = rng.standard_normal((L, d)).astype(np.float32)
    n = sum(sizes)
    owner = np.repeat(np.arange(L), sizes)
    X = (C[owner] + 0.7 * rng.standard_normal((n, d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.7 * rng.standard_normal((nq, d))).astype(np.float32)
    if normalized:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
        C /= np.linalg.norm(C, axis=1, keepdims=True)
    ids = np.arange(n, dtype=np.int64) * 3 + 11
    alive = np.ones(n, np.uint8)
    alive[rng.random(n) < 0.04] = 0
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    return dict(metric=metric, normalized=normalized, C=C, X=X, Q=Q, ids=ids, alive=alive,
                off=off, nprobe=nprobe, k=k)


def search(cabi, case, tile_rows, storage=None):
    e = cabi.Engine()
    d = case["C"].shape[1]
    kw = {} if storage is None else {"storage": storage}
    e.create_ivf(1, d, case["metric"], case["normalized"], case["C"], **kw)
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
    e.set_scan_tile_rows(tile_rows)
    out = e.search(1, case["Q"], case["k"], case["nprobe"])
    e.stop()
    return out


def same(a, b):
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


@pytest.mark.parametrize("name", list(CASES))
def test_row_tiles_change_nothing(cuda_ok, oracle_mod, name):
    from m3_memory_b200 import cabi

    case = make_case(name)
    whole = search(cabi, case, -1)
    tiled = search(cabi, case, 128)
    same(tiled, whole)
    same(search(cabi, case, 384), whole)
    lists = oracle_mod.CsrLists(case["off"], case["X"], case["ids"], case["alive"])
    ref = oracle_mod.search_nprobe(case["Q"], case["C"], lists, case["metric"],
                                   case["normalized"], case["k"], case["nprobe"])
    # the tiling is checked exactly above; against the oracle the scan keeps its
    # usual accuracy (ids may differ only at near-ties at the k-th place: these
    # low-dimensional Gaussian cases have a few within the scan's 2^-16 relative
    # error, so the bar here is 0.995 rather than the 0.999 of realistic data)
    compare_search(tiled, ref, min_recall=0.995)


def test_bf16_rows_in_tiles(cuda_ok):
    from m3_memory_b200 import cabi

    case = make_case("l2_k33")
    whole = search(cabi, case, -1, storage=cabi.BF16)
    same(search(cabi, case, 128, storage=cabi.BF16), whole)


@pytest.mark.parametrize("nq", [24, 64])
def test_automatic_tiles_of_a_wide_index(cuda_ok, oracle_mod, nq):
    """dim 1024 (4 KB rows) with the default setting: 64 queries x 3 probes (more
    pairs than SMs) take tiles of about 4 MB (1024 rows), so the 2600- and
    4500-row lists are tiled; 24 queries x 3 probes (fewer pairs than SMs) take
    128-row tiles, so every list longer than that is."""
    from m3_memory_b200 import cabi

    CASES["ip_wide_auto"] = (1, False, 1024, nq, 3, 10)
    try:
        case = make_case("ip_wide_auto", sizes=[2600, 40, 4500, 700, 0, 1100])
    finally:
        del CASES["ip_wide_auto"]
    whole = search(cabi, case, -1)
    same(search(cabi, case, 0), whole)
    lists = oracle_mod.CsrLists(case["off"], case["X"], case["ids"], case["alive"])
    ref = oracle_mod.search_nprobe(case["Q"], case["C"], lists, case["metric"],
                                   case["normalized"], case["k"], case["nprobe"])
    compare_search(whole, ref, min_recall=0.995)


def test_tiles_beyond_the_region_scan_whole(cuda_ok):
    """60 queries probing every list (two query groups each): the 40000-row list
    would take 313 tiles x 60 pairs, more than the 16384 partial lists of the tile
    region, so it is scanned whole while the 3000-row list is tiled; the answer
    is the same."""
    from m3_memory_b200 import cabi

    CASES["ip_region"] = (1, False, 32, 60, -1, 10)
    try:
        case = make_case("ip_region", sizes=[40000, 3000, 50])
    finally:
        del CASES["ip_region"]
    same(search(cabi, case, 128), search(cabi, case, -1))


def test_tile_rows_argument(cuda_ok):
    from m3_memory_b200 import cabi

    e = cabi.Engine()
    for bad in (-2, 100, 129):
        with pytest.raises(ValueError):
            e.set_scan_tile_rows(bad)
    for ok in (-1, 0, 128, 4096):
        e.set_scan_tile_rows(ok)
