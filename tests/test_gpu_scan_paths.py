"""The tensor-core list scan (the default for inner product and cosine with
k <= 32) against the oracle, and against the SIMT scan (M3G_SCAN=simt, run in a
child process because the choice is read once per process).

The cases exercise the scan's structure: a list longer than one pass of row
blocks (2100 rows), ragged last blocks, a dimension that is not a multiple of
32, empty and tiny lists, erased rows, items of up to 32 queries, k up to
32, and both cosine forms."""
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
