"""Comparison helpers shared by the parity tests.

Tolerances (the parity bar): cluster assignments and nprobe selections are
bit-exact except at exact-score ties; returned top-k ids reach recall >= 0.999
against the reference; returned scores agree with the reference's within
SCORE_RTOL relative error (with SCORE_ATOL absolute floor for scores near 0).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
SCORE_RTOL = 1e-3
SCORE_ATOL = 1e-6
MIN_RECALL = 0.999


def load_golden(name):
    return dict(np.load(GOLDEN / f"{name}.npz"))


INDEX_CASES = ["cosine_norm", "ip_mixture", "l2_raw", "cosine_raw_zero", "edge_k_gt_candidates"]
KMEANS_CASES = ["kmeans_ip", "kmeans_l2"]


def canon(ids, scores, counts):
    """Rows sorted by (score, id) so exactly tied scores compare in one order."""
    ids, scores = ids.copy(), scores.copy()
    for q in range(ids.shape[0]):
        c = int(counts[q])
        o = np.lexsort((ids[q, :c], scores[q, :c]))
        ids[q, :c] = ids[q, :c][o]
        scores[q, :c] = scores[q, :c][o]
    return ids, scores


def _boundary_ties(scores, c, k):
    """Mask of the entries tied exactly with a full row's last (k-th) score:
    which of several equal-score candidates fill the last slots is left open
    by the reference (nth_element / unstable sort / replacement order)."""
    m = np.zeros(c, bool)
    if c == k and c > 0:
        m = scores[:c] == scores[c - 1]
        if m.sum() < 2:
            m[:] = False
    return m


def compare_search(got, ref, rtol=SCORE_RTOL, atol=SCORE_ATOL, min_recall=MIN_RECALL,
                   exact=False):
    """Recall of got's ids against ref's, plus per-id score agreement.

    Returns the recall.  Entries tied exactly at a full row's boundary score in
    the reference count as hits when got's entry carries that score too.
    exact=True demands identical sorted scores and identical ids outside such
    ties (used for oracle-vs-reference checks)."""
    g_ids, g_sc, g_cnt = got
    r_ids, r_sc, r_cnt = ref
    assert g_ids.shape[0] == r_ids.shape[0]
    np.testing.assert_array_equal(g_cnt, r_cnt)
    k = r_ids.shape[1]
    if exact:
        gi, gs = canon(g_ids, g_sc, g_cnt)
        ri, rs = canon(r_ids, r_sc, r_cnt)
        for q in range(gi.shape[0]):
            c = int(r_cnt[q])
            np.testing.assert_array_equal(gs[q, :c], rs[q, :c])
            tie = _boundary_ties(rs[q], c, k)
            assert sorted(gi[q, :c][~tie].tolist()) == sorted(ri[q, :c][~tie].tolist()), q
        return 1.0
    hit = tot = 0
    for q in range(g_ids.shape[0]):
        c = int(r_cnt[q])
        if c == 0:
            continue
        rmap = dict(zip(r_ids[q, :c].tolist(), r_sc[q, :c].tolist()))
        tie = _boundary_ties(r_sc[q], c, k)
        tie_score = float(r_sc[q, c - 1]) if tie.any() else None
        for i, s in zip(g_ids[q, :c].tolist(), g_sc[q, :c].tolist()):
            if i in rmap:
                hit += 1
                rs = rmap[i]
                assert abs(s - rs) <= rtol * abs(rs) + atol, (q, i, s, rs)
            elif tie_score is not None and abs(s - tie_score) <= rtol * abs(tie_score) + atol:
                hit += 1
        tot += c
        # scores come back ascending
        assert np.all(np.diff(g_sc[q, :c]) >= 0), q
    recall = hit / max(tot, 1)
    assert recall >= min_recall, recall
    return recall


def lists_of(g):
    """(off, vecs, ids, alive) of a golden index case."""
    return g["off"], g["lvecs"], g["lids"], g["lalive"]
