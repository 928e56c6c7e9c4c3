"""Indexes whose lists are stored as bf16 (m3g_create_ivf_ex with M3G_BF16).

The reference stores fp32 only (Cluster::mat_, AgentMemory/M3/include/
cluster.h:83), so the oracle is fed the bf16-rounded values widened to fp32:
a bf16 index must answer exactly as the reference does on those values (ids
with recall >= 0.999, scores within 1e-3 relative; squared L2 scores are the
reference's own sums).  Rows reach the index through load_cluster (fp32 or
bf16 input), the writer threads (insert, update, delete), a split and a
save / load round trip."""
import numpy as np
import pytest

from helpers import compare_search

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cabi(cuda_ok):
    from m3_memory_b200 import cabi as c

    return c


def make_lists(rng, L, d, sizes, scale=1.0):
    C = (scale * rng.standard_normal((L, d))).astype(np.float32)
    owner = np.repeat(np.arange(L), sizes)
    X = (C[owner] + 0.6 * rng.standard_normal((len(owner), d))).astype(np.float32)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    return C, X, off


@pytest.mark.parametrize("metric,normalized,d,k,nprobe", [
    (0, False, 768, 100, 4),   # the bf16 configuration: squared L2, dim 768, k 100
    (0, False, 100, 10, 3),    # dim not a multiple of 64
    (1, False, 256, 64, 3),
    (2, True, 128, 10, -1),
    (2, False, 36, 128, 5),    # rows padded to one 64-wide box
])
def test_bf16_lists_match_oracle_on_rounded_values(cabi, oracle_mod, metric, normalized, d, k,
                                                   nprobe):
    O = oracle_mod
    rng = np.random.default_rng(d + k + metric)
    sizes = [0, 7, 140, 333, 1290, 2100, 65, 1]
    L = len(sizes)
    C, X, off = make_lists(rng, L, d, sizes)
    Q = (C[rng.integers(0, L, 48)] + 0.6 * rng.standard_normal((48, d))).astype(np.float32)
    if normalized:
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
        C /= np.linalg.norm(C, axis=1, keepdims=True)
    ids = np.arange(len(X), dtype=np.int64) * 3 + 1
    e = cabi.Engine()
    e.create_ivf(1, d, metric, normalized, C, storage=cabi.BF16)
    assert e.storage_of(1) == cabi.BF16
    for c in range(L):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            # half the lists arrive as fp32 (rounded by the engine), half as bf16 bits
            v = X[b:t] if c % 2 else cabi.bf16_bits(X[b:t])
            e.load_cluster(1, c, ids[b:t], v)
    Xr = cabi.bf16_round(X)
    got = e.search(1, Q, k, nprobe)
    lists = O.CsrLists(off, Xr, ids)
    ref = O.search_nprobe(Q, C, lists, metric, normalized, k, nprobe)
    compare_search(got, ref)
    if metric == 0:
        # squared L2 comes back as the reference's own sum over the stored values
        row_of = {int(i): r for r, i in enumerate(ids)}
        for q in range(len(Q)):
            c = int(got[2][q])
            want = [O.score(Q[q], Xr[row_of[int(i)]], 0, False) for i in got[0][q, :c]]
            np.testing.assert_array_equal(np.array(want, np.float32), got[1][q, :c])
    # the stored rows read back as the rounded values
    gi, gv = e.get_cluster(1, 4)
    np.testing.assert_array_equal(gv, Xr[off[4]:off[5]])


def test_bf16_writes_split_and_persistence(cabi, oracle_mod, tmp_path):
    O = oracle_mod
    rng = np.random.default_rng(12)
    d, L = 192, 6
    sizes = [400, 10, 900, 250, 0, 33]
    C, X, off = make_lists(rng, L, d, sizes, scale=2.0)
    ids = np.arange(len(X), dtype=np.int64)
    e = cabi.Engine()
    e.create_ivf(1, d, 0, False, C, storage=cabi.BF16)
    e.start(2, 0)
    for c in range(L):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            assert e.enqueue_insert(1, c, ids[b:t], X[b:t])
    e.flush()
    # updates (rounded again on the way in), deletes, inserts past the list's capacity
    upd = ids[off[2]:off[2] + 50]
    newv = (X[upd] + 0.1).astype(np.float32)
    assert e.enqueue_update(1, 2, upd, newv)
    dele = ids[off[0]:off[0] + 30]
    assert e.enqueue_delete(1, 0, dele)
    extra_ids = np.arange(10_000, 10_700, dtype=np.int64)
    extra = (C[3] + 0.6 * rng.standard_normal((700, d))).astype(np.float32)
    assert e.enqueue_insert(1, 3, extra_ids, extra)
    e.flush()
    e.stop()
    # the same edits on the host copy (bf16-rounded values)
    Xh = X.copy()
    Xh[upd] = newv
    rows = {c: list(range(int(off[c]), int(off[c + 1]))) for c in range(L)}
    rows[0] = [r for r in rows[0] if r not in set(dele.tolist())]
    allv = np.concatenate([Xh, extra])
    allid = np.concatenate([ids, extra_ids])
    rows[3] += list(range(len(X), len(X) + 700))
    order = [r for c in range(L) for r in rows[c]]
    loff = np.concatenate([[0], np.cumsum([len(rows[c]) for c in range(L)])]).astype(np.int64)
    lists = O.CsrLists(loff, cabi.bf16_round(allv[order]), allid[order])
    Q = (C[rng.integers(0, L, 40)] + 0.6 * rng.standard_normal((40, d))).astype(np.float32)
    ref = O.search_nprobe(Q, C, lists, 0, False, 20, 3)
    compare_search(e.search(1, Q, 20, 3), ref)
    # save / load keeps the storage type and the answers
    path = str(tmp_path / "bf16.m3g")
    e.save_index(1, path)
    e.load_index(2, path)
    assert e.storage_of(2) == cabi.BF16
    a, b = e.search(1, Q, 20, 3), e.search(2, Q, 20, 3)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    # a split runs 2-means on the stored (rounded) values, as the oracle's split
    Xl = cabi.bf16_round(allv[rows[3]])
    C2, side = O.split_2means(Xl, 5, 9, 0, False)
    nid = e.split_cluster(1, 3, niter=5, seed=9)
    assert nid == L
    got = e.centroids(1)
    np.testing.assert_array_equal(got[3], C2[0])
    np.testing.assert_array_equal(got[nid], C2[1])


def test_bf16_limits(cabi):
    e = cabi.Engine()
    C = np.eye(8, 64, dtype=np.float32)
    e.create_ivf(1, 64, 0, False, C, storage=cabi.BF16)
    e.load_cluster(1, 0, np.arange(5), np.ones((5, 64), np.float32))
    with pytest.raises(cabi.M3GError) as ei:
        e.search(1, np.ones((2, 64), np.float32), 129, 2)
    assert ei.value.code == cabi.M3G_EUNSUPPORTED
    with pytest.raises(ValueError):  # M3G_EINVAL
        e.create_ivf(2, 64, 0, False, C, storage=7)


@pytest.mark.parametrize("storage", [0, 1])
def test_device_loading_equals_host_loading(cabi, storage):
    """m3g_load_cluster_device (rows already on the GPU, fp32 or bf16 bits) builds
    the same lists as the host path, and m3g_nearest_clusters_device gives the
    host assignment."""
    import torch

    rng = np.random.default_rng(3 + storage)
    d, L = 100, 5
    sizes = [120, 0, 700, 33, 260]
    C, X, off = make_lists(rng, L, d, sizes)
    ids = np.arange(len(X), dtype=np.int64) + 50
    Q = (C[rng.integers(0, L, 30)] + 0.6 * rng.standard_normal((30, d))).astype(np.float32)
    host, dev = cabi.Engine(), cabi.Engine()
    for e in (host, dev):
        e.create_ivf(1, d, 0, False, C, storage=storage)
    for c in range(L):
        b, t = int(off[c]), int(off[c + 1])
        host.load_cluster(1, c, ids[b:t], X[b:t])
        di = torch.from_numpy(ids[b:t].copy()).cuda()
        if c % 2:
            dv = torch.from_numpy(cabi.bf16_bits(X[b:t])).cuda()
            dev.load_cluster_device(1, c, di.data_ptr(), dv.data_ptr(), t - b, cabi.BF16)
        else:
            dv = torch.from_numpy(X[b:t].copy()).cuda()
            dev.load_cluster_device(1, c, di.data_ptr(), dv.data_ptr(), t - b, cabi.F32)
        torch.cuda.synchronize()
    if storage == 1:
        a, b = host.search(1, Q, 10, 3), dev.search(1, Q, 10, 3)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)
    for c in range(L):
        hi, hv = host.get_cluster(1, c)
        gi, gv = dev.get_cluster(1, c)
        np.testing.assert_array_equal(hi, gi)
        if storage == 1 or c % 2 == 0:
            np.testing.assert_array_equal(hv, gv)
        else:  # fp32 storage of bf16 input holds the bf16 values
            np.testing.assert_array_equal(gv, cabi.bf16_round(hv))
    xd = torch.from_numpy(X).cuda()
    out = torch.empty(len(X), dtype=torch.int32, device="cuda")
    dev.nearest_clusters_device(1, xd.data_ptr(), len(X), out.data_ptr())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), host.nearest_clusters(1, X))


@pytest.mark.parametrize("storage", [0, 1])
def test_one_pass_device_load_equals_list_by_list(cabi, storage):
    """m3g_load_lists_device (every list at once from device rows and their
    assignment, -1 skipping a row) builds the same lists as m3g_load_cluster
    called per list with each list's rows in order, and later inserts grow it."""
    import torch

    rng = np.random.default_rng(31 + storage)
    d, L, n = 72, 9, 3000
    C = rng.standard_normal((L, d)).astype(np.float32)
    a = rng.integers(-1, L, n).astype(np.int32)
    a[a == 4] = 5  # an empty list
    X = (C[np.maximum(a, 0)] + 0.5 * rng.standard_normal((n, d))).astype(np.float32)
    ids = rng.permutation(10 * n)[:n].astype(np.int64)
    one, per = cabi.Engine(), cabi.Engine()
    for e in (one, per):
        e.create_ivf(1, d, 0, False, C, storage=storage)
    for c in range(L):
        rows = np.flatnonzero(a == c)
        per.load_cluster(1, c, ids[rows], X[rows])
    ta, ti, tx = (torch.from_numpy(v).cuda() for v in (a, ids, X))
    one.load_lists_device(1, ta.data_ptr(), ti.data_ptr(), tx.data_ptr(), n)
    torch.cuda.synchronize()
    for c in range(L):
        for u, v in zip(one.get_cluster(1, c), per.get_cluster(1, c)):
            np.testing.assert_array_equal(u, v)
    Q = (C[rng.integers(0, L, 25)] + 0.5 * rng.standard_normal((25, d))).astype(np.float32)
    for u, v in zip(one.search(1, Q, 10, 4), per.search(1, Q, 10, 4)):
        np.testing.assert_array_equal(u, v)
    for e in (one, per):
        e.start(1, 0)
        assert e.enqueue_insert_auto(1, np.arange(10 * n, 10 * n + 500, dtype=np.int64),
                                     (C[rng.integers(0, L, 500) * 0 + 2] + 0.5).astype(np.float32))
        e.flush()
        e.stop()
    for u, v in zip(one.search(1, Q, 10, 4), per.search(1, Q, 10, 4)):
        np.testing.assert_array_equal(u, v)
