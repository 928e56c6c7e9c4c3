"""Generates tests/golden/*.npz by running the reference's own C++ core.

The reference ships no tests, fixtures or known-answer vectors for its IVF
path, so the golden vectors are produced here: seeded synthetic inputs are fed
to the reference core (AgentMemory/M3/src/{base,cluster,m3_index,m3_async}.cpp,
compiled from its sources by oracle/Makefile into oracle/_ref/liboracle_ref.so)
and its outputs are stored next to the inputs.  The k-means fixture has no
reference counterpart: it stores the oracle restatement's result (its E-step
is checked against the reference's nearest_clusters when generated).

Run from the repository root:  python tests/golden/make_golden.py
(needs the reference tree to build liboracle_ref.so; the fixtures then travel
without it).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402
from m3_memory_b200 import synthetic as S  # noqa: E402

OUT = Path(__file__).resolve().parent


def _index_case(name, metric, normalized, n, d, nlist, nq, k, nprobes, seed, data="unit",
                zero_rows=0, dead_frac=0.0, empty_lists=0, dup_rows=0):
    rng = np.random.default_rng(seed)
    if data == "unit":
        X = S.unit_gaussian(n, d, rng)
        Q = S.unit_gaussian(nq, d, rng)
    elif data == "mixture":
        means = S.mixture_means(max(4, nlist // 2), d, rng)
        X, _ = S.gaussian_mixture(n, means, 0.3, rng)
        Q, _ = S.gaussian_mixture(nq, means, 0.3, rng)
    else:  # raw: unnormalised Gaussian rows with varied norms
        X = (rng.standard_normal((n, d)) * rng.uniform(0.2, 3.0, (n, 1))).astype(np.float32)
        Q = (rng.standard_normal((nq, d)) * rng.uniform(0.2, 3.0, (nq, 1))).astype(np.float32)
    if zero_rows:
        X[rng.choice(n, zero_rows, replace=False)] = 0.0
        Q[0] = 0.0
    if dup_rows:
        src = rng.choice(n, dup_rows, replace=False)
        dst = rng.choice(n, dup_rows, replace=False)
        X[dst] = X[src]
    C = X[O.sample_rows(seed + 1, n, nlist)].copy()
    if empty_lists:
        # centroids far from every row: those lists stay empty
        C[-empty_lists:] = 50.0 + rng.standard_normal((empty_lists, d)).astype(np.float32)
    ref = O.RefIndex(d, metric, normalized)
    ref.set_centroids(C)
    assign = ref.nearest_clusters(X)
    ids = (np.arange(n, dtype=np.int64) * 7 + 3)
    lists = O.CsrLists.from_assign(X, ids, assign, nlist)
    alive = np.ones(n, np.uint8)
    if dead_frac:
        alive[rng.random(n) < dead_frac] = 0
    lists.alive = alive
    lists.to_ref(ref)
    out = dict(metric=metric, normalized=int(normalized), Q=Q, C=C,
               assign=assign, off=lists.off, lvecs=lists.vecs, lids=lists.ids,
               lalive=lists.alive, k=k, nprobes=np.array(nprobes, np.int32))
    for p in nprobes:
        r_ids, r_sc, r_cnt = ref.search_nprobe(Q, k, p)
        out[f"ref_ids_p{p}"] = r_ids
        out[f"ref_scores_p{p}"] = r_sc
        out[f"ref_counts_p{p}"] = r_cnt
    np.savez_compressed(OUT / f"{name}.npz", **out)
    print("wrote", name)


def _kmeans_case(name, metric, normalized, n, d, nlist, niter, seed):
    rng = np.random.default_rng(seed)
    means = S.mixture_means(nlist, d, rng)
    X, _ = S.gaussian_mixture(n, means, 0.4, rng)
    C, a = O.kmeans_train(X, nlist, niter, seed, metric, normalized)
    ref = O.RefIndex(d, metric, normalized)
    ref.set_centroids(C)
    assert (ref.nearest_clusters(X) == a).all()
    C2, a2 = O.split_2means(X[a == 0], 5, seed + 7, metric, normalized)
    np.savez_compressed(OUT / f"{name}.npz", metric=metric, normalized=int(normalized), X=X,
                        nlist=nlist, niter=niter, seed=seed, C=C, assign=a, split_C=C2,
                        split_assign=a2, split_seed=seed + 7)
    print("wrote", name)


def main():
    O.build(ref=True)
    _index_case("cosine_norm", O.COSINE, True, 1500, 64, 16, 40, 10, [4, 0, 32], seed=11)
    _index_case("ip_mixture", O.IP, False, 1500, 96, 24, 40, 10, [3, 8], seed=12, data="mixture")
    _index_case("l2_raw", O.L2, False, 1200, 40, 12, 30, 7, [2, 5], seed=13, data="raw",
                dead_frac=0.1)
    _index_case("cosine_raw_zero", O.COSINE, False, 1000, 36, 10, 30, 12, [3], seed=14,
                data="raw", zero_rows=5)
    _index_case("edge_k_gt_candidates", O.L2, False, 300, 32, 20, 20, 64, [1, 2], seed=15,
                empty_lists=4, dup_rows=20)
    _kmeans_case("kmeans_ip", O.IP, False, 2000, 48, 12, 6, seed=21)
    _kmeans_case("kmeans_l2", O.L2, False, 1500, 24, 9, 5, seed=22)


if __name__ == "__main__":
    main()
