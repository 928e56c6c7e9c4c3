"""The exact top-P selection across its block shapes and paths, against the
oracle's select_nprobe (the reference's SelectNprobe order: ascending exact
score, ties by lower id).

P runs over both block shapes (the small one takes P <= 128, the large one
the rest), over the pre-filtered threshold (P <= 128) and the general path,
and past 1024 (ids returned unsorted).  The centroid sets cover a clustered
mixture (close scores: most candidates are rescored), more centroids than the
shared-memory key caches hold (L = 9000), and near-duplicate centroids whose
intervals all overlap (S0 and the candidate list overflow into the exact
fallback), and centroids stored twice each, whose intervals overlap in pairs
among more than 128 candidates (the sorted overlap test).  The same cases run
through the set form of the selection (membership only)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# name: metric (0 L2, 1 IP, 2 COSINE), normalized, L, dim, nq, P values
CASES = {
    "ip_mixture": (1, False, 2048, 256, 48, (1, 8, 32, 64, 100, 128, 129, 256, 1024, 1500)),
    "l2_mixture": (0, False, 2048, 96, 32, (1, 32, 128, 200)),
    "cos_raw": (2, False, 1500, 130, 32, (1, 32, 127, 300)),
    "cos_norm_wide": (2, True, 9000, 64, 24, (1, 16, 64, 128, 500)),
    "ip_near_duplicates": (1, False, 600, 128, 16, (1, 8, 64, 128, 400)),
    "l2_duplicate_pairs": (0, False, 1000, 64, 16, (129, 200, 256, 700)),
    # centroid norms from 0.14 to 7.4: the first pass's uniform norm bound (the
    # largest norm) is far wider than most centroids' own
    "ip_varied_norms": (1, False, 2048, 256, 32, (1, 8, 32, 128, 256)),
}


def make_case(name):
    metric, normalized, L, d, nq, _ = CASES[name]
    rng = np.random.default_rng(sum(map(ord, name)))
    if name == "ip_near_duplicates":
        base = rng.standard_normal(d).astype(np.float32)
        C = (base + 1e-6 * rng.standard_normal((L, d))).astype(np.float32)
        C[::7] = base  # exact duplicates: exact ties, broken by id
        Q = (base + 0.5 * rng.standard_normal((nq, d))).astype(np.float32)
    elif name == "l2_duplicate_pairs":
        # every centroid twice (ids 2i and 2i + 1): many overlapping pairs of
        # intervals among candidates that are otherwise well apart, the case the
        # sorted overlap test (more than 128 candidates) must flag exactly
        U = (4.0 * rng.standard_normal((L // 2, d))).astype(np.float32)
        C = np.repeat(U, 2, axis=0)
        Q = (U[rng.integers(0, L // 2, nq)] + rng.standard_normal((nq, d))).astype(np.float32)
    else:
        means = rng.standard_normal((16, d)).astype(np.float32)
        C = (means[rng.integers(0, 16, L)] + 0.3 * rng.standard_normal((L, d))).astype(np.float32)
        Q = (means[rng.integers(0, 16, nq)] + 0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    if name == "ip_varied_norms":
        C *= np.exp(rng.uniform(-2.0, 2.0, (L, 1))).astype(np.float32)
    if normalized:
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return metric, normalized, C, Q


@pytest.mark.parametrize("name", list(CASES))
def test_select_matches_oracle(cuda_ok, oracle_mod, name):
    from m3_memory_b200 import cabi

    O = oracle_mod
    metric, normalized, C, Q = make_case(name)
    e = cabi.Engine()
    e.create_ivf(1, C.shape[1], metric, normalized, C)
    for p in CASES[name][5]:
        got = e.select_probes(1, Q, p)
        pp = min(p, len(C))
        assert got.shape == (len(Q), pp), (name, p, got.shape)
        for q in range(len(Q)):
            want = O.select_nprobe(Q[q], C, metric, normalized, p)
            if pp > 1024:
                # above 1024 the set is returned in ascending id order
                np.testing.assert_array_equal(np.sort(got[q]), np.sort(want), err_msg=f"{name} P={p} q={q}")
                np.testing.assert_array_equal(got[q], np.sort(got[q]))
            else:
                np.testing.assert_array_equal(got[q], want, err_msg=f"{name} P={p} q={q}")


@pytest.mark.parametrize("name", list(CASES))
def test_probe_sets_match_oracle(cuda_ok, oracle_mod, name):
    """m3g_select_probe_sets_device (the form the search's scan consumes: only
    the centroids near the P-th place are rescored) returns, per query, exactly
    the oracle's selected set, without repeats, and the same rows on a second
    call.  Batches of 1 and 5 take the GEMV coarse step, the full batch the GEMM."""
    import torch

    from m3_memory_b200 import cabi

    O = oracle_mod
    metric, normalized, C, Q = make_case(name)
    e = cabi.Engine()
    e.create_ivf(1, C.shape[1], metric, normalized, C)
    for p in CASES[name][5]:
        pp = min(p, len(C))
        want = [np.sort(O.select_nprobe(Q[q], C, metric, normalized, p)) for q in range(len(Q))]
        for nq in sorted({1, 5, len(Q)}):
            dq = torch.from_numpy(np.ascontiguousarray(Q[:nq])).cuda()
            out = torch.full((nq, pp), -7, dtype=torch.int32, device="cuda")
            e.select_probe_sets_device(1, dq.data_ptr(), nq, p, out.data_ptr())
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            again = torch.full_like(out, -7)
            e.select_probe_sets_device(1, dq.data_ptr(), nq, p, again.data_ptr())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(again.cpu().numpy(), got, err_msg=f"{name} P={p}")
            for q in range(nq):
                np.testing.assert_array_equal(np.sort(got[q]), want[q],
                                              err_msg=f"{name} P={p} nq={nq} q={q}")


@pytest.mark.parametrize("metric,normalized,d", [(1, False, 256), (0, False, 1024),
                                                 (2, False, 2000), (2, True, 96)])
def test_tiny_batches_select_like_the_oracle(cuda_ok, oracle_mod, metric, normalized, d):
    """Batches of 1 to 8 queries take the GEMV coarse step (every SM streams the
    centroids once; the SIMT GEMM's error bound); their selections must be the
    oracle's, as the larger batches' are.  At dim 2000 eight queries exceed the
    GEMV's shared-memory stage and take the GEMM, one query the GEMV."""
    from m3_memory_b200 import cabi

    O = oracle_mod
    rng = np.random.default_rng(d + metric)
    L = 1500
    means = rng.standard_normal((16, d)).astype(np.float32)
    C = (means[rng.integers(0, 16, L)] + 0.3 * rng.standard_normal((L, d))).astype(np.float32)
    Q = (means[rng.integers(0, 16, 8)] + 0.3 * rng.standard_normal((8, d))).astype(np.float32)
    if normalized:
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    e = cabi.Engine()
    e.create_ivf(1, d, metric, normalized, C)
    for nq in (1, 3, 8):
        for p in (1, 16, 200):
            got = e.select_probes(1, Q[:nq], p)
            for q in range(nq):
                want = O.select_nprobe(Q[q], C, metric, normalized, p)
                np.testing.assert_array_equal(got[q], want, err_msg=f"nq={nq} P={p} q={q}")


@pytest.mark.parametrize("metric,normalized,d", [(1, False, 128), (0, False, 96),
                                                 (2, False, 64), (2, True, 200)])
def test_tiny_batches_over_many_centroids(cuda_ok, oracle_mod, metric, normalized, d):
    """1 to 8 queries over 5000 centroids (the GEMV coarse step) select exactly
    the oracle's P ids, with exact duplicate centroids far apart in id (ties broken
    by the lower id) and P from 1 to 128; a batch of 12 (the GEMM coarse step, a
    different error bound and candidate set) agrees with them."""
    from m3_memory_b200 import cabi

    O = oracle_mod
    rng = np.random.default_rng(7 * d + metric)
    L = 5000
    means = rng.standard_normal((24, d)).astype(np.float32)
    C = (means[rng.integers(0, 24, L)] + 0.3 * rng.standard_normal((L, d))).astype(np.float32)
    C[[100, 700, 1300, 4999]] = C[5]  # exact duplicates in several parts
    Q = (means[rng.integers(0, 24, 12)] + 0.3 * rng.standard_normal((12, d))).astype(np.float32)
    Q[0] = C[5]
    if normalized:
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    e = cabi.Engine()
    e.create_ivf(1, d, metric, normalized, C)
    for p in (1, 8, 100, 128):
        big = e.select_probes(1, Q, p)
        for nq in (1, 5, 8):
            got = e.select_probes(1, Q[:nq], p)
            np.testing.assert_array_equal(got, big[:nq], err_msg=f"nq={nq} P={p}")
            for q in range(nq):
                want = O.select_nprobe(Q[q], C, metric, normalized, p)
                np.testing.assert_array_equal(got[q], want, err_msg=f"nq={nq} P={p} q={q}")


@pytest.mark.parametrize("metric,normalized", [(1, False), (2, True)])
def test_select_after_centroid_updates(cuda_ok, oracle_mod, metric, normalized):
    """The selection's uniform norm bound follows set_centroid and add_cluster:
    a centroid moved far out (the new largest norm), one shrunk, and a new
    cluster, then both selection forms against the oracle on the updated
    centroids (for normalised cosine the new rows are unit vectors)."""
    import torch

    from m3_memory_b200 import cabi

    O = oracle_mod
    rng = np.random.default_rng(7 + metric)
    L, d, nq, P = 600, 128, 24, 16
    means = rng.standard_normal((8, d)).astype(np.float32)
    C = (means[rng.integers(0, 8, L)] + 0.3 * rng.standard_normal((L, d))).astype(np.float32)
    Q = (means[rng.integers(0, 8, nq)] + 0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    if normalized:
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    e = cabi.Engine()
    e.create_ivf(1, d, metric, normalized, C)
    e.select_probes(1, Q, P)
    big = (Q[0] * (1.0 if normalized else 9.0)).astype(np.float32)
    small = (C[5] * (1.0 if normalized else 0.05)).astype(np.float32)
    extra = (Q[3] + 0.01 * rng.standard_normal(d)).astype(np.float32)
    if normalized:
        extra /= np.linalg.norm(extra)
    e.set_centroid(1, 17, big)
    e.set_centroid(1, 5, small)
    e.add_cluster(1, extra)
    C2 = np.concatenate([C, extra[None]]).astype(np.float32)
    C2[17], C2[5] = big, small
    got = e.select_probes(1, Q, P)
    dq = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    out = torch.full((nq, P), -7, dtype=torch.int32, device="cuda")
    e.select_probe_sets_device(1, dq.data_ptr(), nq, P, out.data_ptr())
    torch.cuda.synchronize()
    sets = out.cpu().numpy()
    for q in range(nq):
        want = O.select_nprobe(Q[q], C2, metric, normalized, P)
        np.testing.assert_array_equal(got[q], want, err_msg=f"q={q}")
        np.testing.assert_array_equal(np.sort(sets[q]), np.sort(want), err_msg=f"set q={q}")
