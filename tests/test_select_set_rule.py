"""The membership rule of the set form of the exact selection, restated on the
host and checked against the true top-P on random intervals.

Every centroid c has an exact score s_c inside a known interval [lo_c, hi_c]
(the GEMM's approximation and its error bound); the top-P set is the P
smallest (s_c, c).  The kernel (select_probes_kernel with kSelectSetOnly)
takes T = the P-th smallest upper bound and the candidates lo_c <= T, then
classifies each candidate: in for certain when fewer than P other candidates
have lo <= its hi, out for certain when at least P others have hi < its lo,
else rescored; the set is the in-for-certain ones plus the best P - (that
many) rescored ones by (s, id).  This test checks that rule, with exact ties,
zero-width intervals and intervals that all overlap, against sorting by
(s, id); it runs without a GPU."""
import numpy as np
import pytest


def set_by_rule(lo, hi, s, P):
    L = len(s)
    T = np.sort(hi)[P - 1]
    cand = np.flatnonzero(lo <= T)
    lo_c, hi_c = lo[cand], hi[cand]
    maybe = (lo_c[None, :] <= hi_c[:, None]).sum(1) - (lo_c <= hi_c)
    surely = (hi_c[None, :] < lo_c[:, None]).sum(1) - (hi_c < lo_c)
    sure_in = cand[maybe < P]
    out = (maybe >= P) & (surely >= P)
    rescored = cand[~(maybe < P) & ~out]
    assert len(rescored) >= P - len(sure_in)
    best = sorted(rescored.tolist(), key=lambda c: (s[c], c))[: P - len(sure_in)]
    return set(sure_in.tolist()) | set(best), len(rescored)


@pytest.mark.parametrize("seed", range(6))
def test_rule_returns_the_true_top_p(seed):
    rng = np.random.default_rng(seed)
    for _ in range(400):
        L = int(rng.integers(1, 300))
        P = int(rng.integers(1, L + 1))
        scale = rng.choice([0.01, 1.0])
        s = np.round(rng.standard_normal(L) * scale, int(rng.choice([2, 6])))  # ties
        w = rng.random(L) * rng.choice([0.0, 1e-3, 5e-2, 10.0])  # up to all overlapping
        lo = s - w * rng.random(L)
        hi = s + w * rng.random(L)
        got, _ = set_by_rule(lo, hi, s, P)
        want = set(sorted(range(L), key=lambda c: (s[c], c))[:P])
        assert got == want


def test_narrow_intervals_rescore_only_the_boundary():
    """With intervals narrower than the gaps around the P-th place only the
    candidates whose intervals reach across it are rescored."""
    rng = np.random.default_rng(11)
    s = np.sort(rng.standard_normal(4096)) * 0.03
    w = np.full(4096, 1e-5)
    rng.shuffle(s)
    _, n = set_by_rule(s - w, s + w, s, 32)
    assert n <= 4
