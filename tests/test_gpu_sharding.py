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


@pytest.mark.parametrize("ns,nq,k", [(2, 50, 10), (8, 33, 7), (3, 5, 1), (4, 9, 64)])
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
