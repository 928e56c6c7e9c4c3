"""The GPU side of list sharding, on one GPU.

* m3g_merge_shards_device against the oracle's restatement of the shard-merge
  rule on random per-shard answers with exact ties, NaN, padding and short rows.
* Two engines on one GPU, each holding the lists one rank of a world of 2 owns
  (m3_memory_b200.sharding.shard_lists), searched separately and merged by the
  merge kernel: equal to one engine holding every list.  This is the multi-GPU
  path with the NCCL all-gather replaced by stacking the two answers."""
import numpy as np
import pytest
import zlib

from helpers import compare_search

pytestmark = pytest.mark.gpu


def _merge_device(cabi, torch, sc, ids):
    e = cabi.Engine()
    ns, nq, k = sc.shape
    d_sc = torch.from_numpy(np.ascontiguousarray(sc)).cuda()
    d_ids = torch.from_numpy(np.ascontiguousarray(ids)).cuda()
    o_ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    o_sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    o_cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
    e.merge_shards_device(d_sc.data_ptr(), d_ids.data_ptr(), ns, nq, k, o_ids.data_ptr(),
                          o_sc.data_ptr(), o_cnt.data_ptr())
    torch.cuda.synchronize()
    return o_ids.cpu().numpy(), o_sc.cpu().numpy(), o_cnt.cpu().numpy()


# (16, 20, 32): 512 candidates per query, the most the warp-per-query merge takes;
# (17, 20, 32) and k = 64 take the block merge
@pytest.mark.parametrize("ns,nq,k", [(2, 50, 10), (8, 33, 7), (3, 5, 1), (4, 9, 64),
                                     (16, 20, 32), (17, 20, 32)])
def test_merge_kernel_matches_rule(cuda_ok, oracle_mod, ns, nq, k):
    import torch

    from m3_memory_b200 import cabi

    rng = np.random.default_rng(ns * 1000 + k)
    sc = np.sort(rng.integers(0, 20, (ns, nq, k)).astype(np.float32) / 8, axis=2)  # many ties
    ids = rng.integers(0, 10**9, (ns, nq, k)).astype(np.int64)
    cnt = rng.integers(0, k + 1, (ns, nq))  # short shard answers: +inf / -1 padding
    for s in range(ns):
        for q in range(nq):
            sc[s, q, cnt[s, q]:] = np.inf
            ids[s, q, cnt[s, q]:] = -1
    sc[0, 0, 0] = np.nan
    got = _merge_device(cabi, torch, sc, ids)
    want = oracle_mod.merge_shards(sc, ids)
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("ns,nq,k", [(2, 50, 10), (3, 7, 3), (4, 9, 64)])
def test_packed_records_merge_as_separate_arrays(cuda_ok, oracle_mod, ns, nq, k):
    """One gathered buffer of answer records ([nq, k] scores, padded to 8 bytes,
    then [nq, k] ids per shard, the layout ShardedSearch all-gathers) merges
    exactly as the separate arrays do."""
    import torch

    from m3_memory_b200 import cabi

    rng = np.random.default_rng(ns * 77 + k)
    sc = np.sort(rng.integers(0, 30, (ns, nq, k)).astype(np.float32) / 4, axis=2)
    ids = rng.integers(0, 10**12, (ns, nq, k)).astype(np.int64)
    sc[:, 1, k // 2:] = np.inf
    ids[:, 1, k // 2:] = -1
    off = (nq * k * 4 + 7) // 8 * 8
    R = off + nq * k * 8
    buf = np.zeros(ns * R, np.uint8)
    for r in range(ns):
        buf[r * R:r * R + nq * k * 4] = sc[r].reshape(-1).view(np.uint8)
        buf[r * R + off:r * R + off + nq * k * 8] = ids[r].reshape(-1).view(np.uint8)
    e = cabi.Engine()
    d = torch.from_numpy(buf).cuda()
    o_ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    o_sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    o_cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
    e.merge_shards_packed_device(d.data_ptr(), ns, nq, k, R, off, o_ids.data_ptr(),
                                 o_sc.data_ptr(), o_cnt.data_ptr())
    torch.cuda.synchronize()
    want = oracle_mod.merge_shards(sc, ids)
    for a, b in zip((o_ids.cpu().numpy(), o_sc.cpu().numpy(), o_cnt.cpu().numpy()), want):
        np.testing.assert_array_equal(a, b)
    with pytest.raises(ValueError):  # a record too short for its ids
        e.merge_shards_packed_device(d.data_ptr(), ns, nq, k, off, off, o_ids.data_ptr(),
                                     o_sc.data_ptr(), o_cnt.data_ptr())


def test_two_shards_on_one_gpu_equal_one_engine(cuda_ok):
    import torch

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import shard_lists

    rng = np.random.default_rng(zlib.crc32(b"shards"))
    L, d, nq, k, nprobe = 40, 96, 64, 10, 12
    sizes = (rng.zipf(1.5, L) * 37) % 700
    C = rng.standard_normal((L, d)).astype(np.float32)
    owner_row = np.repeat(np.arange(L), sizes)
    X = (C[owner_row] + 0.6 * rng.standard_normal((len(owner_row), d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.6 * rng.standard_normal((nq, d))).astype(np.float32)
    ids = np.arange(len(X), dtype=np.int64) + 100
    off = np.concatenate([[0], np.cumsum(sizes)])
    owner = shard_lists(sizes, 2)

    def engine(keep):
        e = cabi.Engine()
        e.create_ivf(1, d, cabi.IP, False, C)
        for c in range(L):
            b, t = int(off[c]), int(off[c + 1])
            if t > b and keep(c):
                e.load_cluster(1, c, ids[b:t], X[b:t])
        return e

    full = engine(lambda c: True).search(1, Q, k, nprobe)
    parts = [engine(lambda c, r=r: owner[c] == r).search(1, Q, k, nprobe) for r in range(2)]
    g_ids = np.stack([p[0] for p in parts])
    g_sc = np.stack([p[1] for p in parts])
    merged = _merge_device(cabi, torch, g_sc, g_ids)
    compare_search(merged, full, exact=True)


def _index_case(seed, L=40, d=96, nq=64, metric=1, normalized=False):
    rng = np.random.default_rng(seed)
    sizes = (rng.zipf(1.5, L) * 37) % 700
    C = rng.standard_normal((L, d)).astype(np.float32)
    owner_row = np.repeat(np.arange(L), sizes)
    X = (C[owner_row] + 0.6 * rng.standard_normal((len(owner_row), d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.6 * rng.standard_normal((nq, d))).astype(np.float32)
    if normalized:
        for a in (C, X, Q):
            a /= np.linalg.norm(a, axis=1, keepdims=True)
    ids = np.arange(len(X), dtype=np.int64) + 100
    off = np.concatenate([[0], np.cumsum(sizes)])
    return dict(C=C, X=X, Q=Q, ids=ids, off=off, sizes=sizes, metric=metric,
                normalized=normalized)


def _engine(cabi, c, keep_list, coarse_ids=None):
    """Index 1: every centroid, the kept lists; index 2 (optional): the
    centroids coarse_ids only (local ids 0..)."""
    e = cabi.Engine()
    d = c["C"].shape[1]
    e.create_ivf(1, d, c["metric"], c["normalized"], c["C"])
    for l in range(len(c["C"])):
        b, t = int(c["off"][l]), int(c["off"][l + 1])
        if t > b and keep_list(l):
            e.load_cluster(1, l, c["ids"][b:t], c["X"][b:t])
    if coarse_ids is not None and len(coarse_ids):
        e.create_ivf(2, d, c["metric"], c["normalized"], c["C"][coarse_ids])
    return e


def test_probe_entry_points(cuda_ok, oracle_mod):
    import torch

    from m3_memory_b200 import cabi

    for metric, norm in ((1, False), (0, False), (2, True), (2, False)):
        c = _index_case(7 + metric, metric=metric, normalized=norm)
        e = _engine(cabi, c, lambda l: True)
        nq, P, k = len(c["Q"]), 9, 10
        q = torch.from_numpy(c["Q"]).cuda()
        # device selection == host selection
        dp = torch.empty((nq, P), dtype=torch.int32, device="cuda")
        e.select_probes_device(1, q.data_ptr(), nq, P, dp.data_ptr())
        np.testing.assert_array_equal(dp.cpu().numpy(), e.select_probes(1, c["Q"], P))
        # exact pair scores == the oracle's unified score, bit for bit; -1 / out of range: inf
        probes = dp.clone()
        probes[0, 0] = -1
        probes[1, 1] = 10**6
        ds = torch.empty((nq, P), dtype=torch.float32, device="cuda")
        e.probe_scores_device(1, q.data_ptr(), nq, probes.data_ptr(), P, ds.data_ptr())
        got = ds.cpu().numpy()
        pr = probes.cpu().numpy()
        for i in range(nq):
            for j in range(P):
                want = (oracle_mod.score(c["Q"][i], c["C"][pr[i, j]], metric, norm)
                        if 0 <= pr[i, j] < len(c["C"]) else np.inf)
                assert got[i, j] == np.float32(want), (i, j, got[i, j], want)
        # search over the engine's own probes == search; with slots skipped == the
        # oracle over the remaining lists
        o_ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        o_sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        o_cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
        e.search_probes_device(1, q.data_ptr(), nq, k, dp.data_ptr(), P, o_ids.data_ptr(),
                               o_sc.data_ptr(), o_cnt.data_ptr())
        got = (o_ids.cpu().numpy(), o_sc.cpu().numpy(), o_cnt.cpu().numpy())
        compare_search(got, e.search(1, c["Q"], k, P), exact=True)
        skip = dp.clone()
        skip[:, 1::2] = -1  # every other slot
        e.search_probes_device(1, q.data_ptr(), nq, k, skip.data_ptr(), P, o_ids.data_ptr(),
                               o_sc.data_ptr(), o_cnt.data_ptr())
        sk = skip.cpu().numpy()
        lists = oracle_mod.CsrLists(c["off"], c["X"], c["ids"])
        refs = [oracle_mod.search_on(c["Q"][i:i + 1], lists,
                                     np.array([int(x) for x in sk[i] if x >= 0], np.int32),
                                     metric, norm, k) for i in range(nq)]
        ref = tuple(np.concatenate([r[j] for r in refs]) for j in range(3))
        # GPU scores differ from the reference's sequential sums by rounding only
        compare_search((o_ids.cpu().numpy(), o_sc.cpu().numpy(), o_cnt.cpu().numpy()), ref)


def test_sharded_coarse_two_engines_equal_one(cuda_ok):
    """The sharded-coarse steps for a world of 2, each rank an engine on this GPU."""
    import torch

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import shard_lists

    c = _index_case(zlib.crc32(b"coarse"))
    L, nq, k, P = len(c["C"]), len(c["Q"]), 10, 12
    owner = shard_lists(c["sizes"], 2)
    q = torch.from_numpy(c["Q"]).cuda()
    cand_sc, cand_id, engines = [], [], []
    for r in range(2):
        own = np.flatnonzero(owner == r)
        e = _engine(cabi, c, lambda l, r=r: owner[l] == r, own)
        engines.append(e)
        pl = min(P, len(own))
        loc = torch.empty((nq, pl), dtype=torch.int32, device="cuda")
        sc = torch.empty((nq, pl), dtype=torch.float32, device="cuda")
        e.select_probes_device(2, q.data_ptr(), nq, pl, loc.data_ptr())
        e.probe_scores_device(2, q.data_ptr(), nq, loc.data_ptr(), pl, sc.data_ptr())
        s_pad = torch.full((nq, P), float("inf"), device="cuda")
        i_pad = torch.full((nq, P), -1, dtype=torch.int64, device="cuda")
        s_pad[:, :pl] = sc
        i_pad[:, :pl] = torch.from_numpy(own).cuda()[loc.long()]
        cand_sc.append(s_pad)
        cand_id.append(i_pad)
    top = _merge_device(cabi, torch, torch.stack(cand_sc).cpu().numpy(),
                        torch.stack(cand_id).cpu().numpy())
    full = _engine(cabi, c, lambda l: True)
    np.testing.assert_array_equal(top[0], full.select_probes(1, c["Q"], P))  # global top-P
    parts = []
    for r, e in enumerate(engines):
        t = torch.from_numpy(top[0]).cuda()
        mine = torch.from_numpy(owner).cuda()[t] == r
        probes = torch.where(mine, t, torch.full_like(t, -1)).to(torch.int32)
        ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
        e.search_probes_device(1, q.data_ptr(), nq, k, probes.data_ptr(), P, ids.data_ptr(),
                               sc.data_ptr(), cnt.data_ptr())
        parts.append((ids.cpu().numpy(), sc.cpu().numpy()))
    merged = _merge_device(cabi, torch, np.stack([p[1] for p in parts]),
                           np.stack([p[0] for p in parts]))
    compare_search(merged, full.search(1, c["Q"], k, P), exact=True)


def test_split_coarse_two_engines_equal_one(cuda_ok):
    """The query-split coarse steps for a world of 3 (odd split of 64 queries), each
    rank an engine on this GPU: every rank selects the probes of its query slice over
    all centroids, the slices are concatenated (the all-gather), every rank scans its
    own lists for all queries, and the shard merge gives the one-engine answer; a
    one-rank ShardedSearch in this mode equals the plain search."""
    import torch

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import ShardedSearch, shard_lists

    c = _index_case(zlib.crc32(b"split"))
    nq, k, P, world = len(c["Q"]), 10, 9, 3
    owner = shard_lists(c["sizes"], world)
    q = torch.from_numpy(c["Q"]).cuda()
    engines = [_engine(cabi, c, lambda l, r=r: owner[l] == r) for r in range(world)]
    chunk = -(-nq // world)
    slices = []
    for r, e in enumerate(engines):
        q0, q1 = min(nq, r * chunk), min(nq, (r + 1) * chunk)
        loc = torch.full((chunk, P), -1, dtype=torch.int32, device="cuda")
        if q1 > q0:
            e.select_probes_device(1, q.data_ptr() + q0 * q.stride(0) * 4, q1 - q0, P,
                                   loc.data_ptr())
        slices.append(loc)
    probes = torch.cat(slices)[:nq].contiguous()
    full = _engine(cabi, c, lambda l: True)
    np.testing.assert_array_equal(probes.cpu().numpy(), full.select_probes(1, c["Q"], P))
    parts = []
    for e in engines:
        ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
        e.search_probes_device(1, q.data_ptr(), nq, k, probes.data_ptr(), P, ids.data_ptr(),
                               sc.data_ptr(), cnt.data_ptr())
        parts.append((ids.cpu().numpy(), sc.cpu().numpy()))
    merged = _merge_device(cabi, torch, np.stack([p[1] for p in parts]),
                           np.stack([p[0] for p in parts]))
    want = full.search(1, c["Q"], k, P)
    compare_search(merged, want, exact=True)
    ss = ShardedSearch(full, 1, k, nq, 1, "cuda", split_coarse=True)
    ss.marks = []  # per-phase events, as bench.py records them for N > 1
    ids, sc, cnt = ss.search(q, P)
    torch.cuda.synchronize()
    compare_search((ids.cpu().numpy(), sc.cpu().numpy(), cnt.cpu().numpy()), want, exact=True)
    assert [n for n, _ in ss.marks] == ["start", "coarse", "probe_exchange", "search"]
    assert all(a.elapsed_time(b) >= 0 for (_, a), (_, b) in zip(ss.marks, ss.marks[1:]))
    # the serving form on one rank is the plain search of the rank's batch
    ids, sc, cnt = ShardedSearch(full, 1, k, nq, 1, "cuda").search_own_batch(q, P)
    torch.cuda.synchronize()
    compare_search((ids.cpu().numpy(), sc.cpu().numpy(), cnt.cpu().numpy()), want, exact=True)


_NCCL_CHILD = r"""
import os, sys, numpy as np, torch, torch.distributed as dist, datetime
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
from m3_memory_b200 import cabi
from m3_memory_b200.sharding import ShardedSearch, shard_lists
import test_gpu_sharding as T
c = T._index_case(5)
owner = shard_lists(c["sizes"], world)
own = np.flatnonzero(owner == rank)
e = T._engine(cabi, c, lambda l: owner[l] == rank, own)
q = torch.from_numpy(c["Q"]).cuda()
out = {}
for name, kw in (("replicated", {}), ("sharded", dict(coarse_index_id=2, owner=owner, rank=rank)),
                 ("split", dict(split_coarse=True, rank=rank))):
    ss = ShardedSearch(e, 1, 10, len(c["Q"]), world, "cuda", **kw)
    ids, sc, cnt = ss.search(q, 12)
    torch.cuda.synchronize()
    out[name + "_ids"], out[name + "_sc"], out[name + "_cnt"] = (
        ids.cpu().numpy(), sc.cpu().numpy(), cnt.cpu().numpy())
B = len(c["Q"]) // world  # serving form: each rank brings its own half of the queries
ss = ShardedSearch(e, 1, 10, B, world, "cuda", rank=rank, timeout_s=60.0)  # host-side limit
ids, sc, cnt = ss.search_own_batch(q[rank * B:(rank + 1) * B].contiguous(), 12)
torch.cuda.synchronize()
g = [torch.empty_like(t) for t in (ids, sc, cnt) for _ in range(world)]
for j, t in enumerate((ids, sc, cnt)):
    dist.all_gather(g[j * world:(j + 1) * world], t.contiguous())
out["own_ids"], out["own_sc"], out["own_cnt"] = (
    torch.cat(g[j * world:(j + 1) * world]).cpu().numpy() for j in range(3))
if rank == 0:
    np.savez(sys.argv[2], **out)
dist.barrier()
dist.destroy_process_group()
"""


def test_sharded_search_over_nccl_two_gpus(cuda_ok, tmp_path):
    import os
    import socket
    import subprocess
    import sys

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from m3_memory_b200 import cabi

    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    f = tmp_path / "nccl.npz"
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", _NCCL_CHILD, root, str(f)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    for p in procs:
        _, err = p.communicate(timeout=300)
        assert p.returncode == 0, err[-2000:]
    got = np.load(f)
    c = _index_case(5)
    full = _engine(cabi, c, lambda l: True).search(1, c["Q"], 10, 12)
    for name in ("replicated", "sharded", "split"):
        compare_search((got[name + "_ids"], got[name + "_sc"], got[name + "_cnt"]), full,
                       exact=True)
    B = len(c["Q"]) // 2  # each rank's own batch, concatenated in rank order
    compare_search((got["own_ids"], got["own_sc"], got["own_cnt"]),
                   tuple(a[:2 * B] for a in full), exact=True)
