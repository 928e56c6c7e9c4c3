"""List sharding on CPU with world size 2 over gloo (no GPU).

Each rank owns the lists m3_memory_b200.sharding.shard_lists gives it, searches
only those lists with the oracle (the reference's algorithm, replicated coarse
selection), the per-rank answers are all-gathered and merged by the shard-merge
rule; the merged answer must equal the unsharded search.  This is the
decomposition the GPU path uses (search per rank, all-gather, merge kernel)."""
import datetime
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

from helpers import compare_search

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=3):
    rng = np.random.default_rng(seed)
    L, d, nq, k, nprobe = 24, 40, 30, 7, 6
    sizes = np.minimum((60 * rng.zipf(1.6, L)) % 400, 400)
    sizes[[3, 11]] = 0  # empty lists
    C = rng.standard_normal((L, d)).astype(np.float32)
    owner_of_row = np.repeat(np.arange(L), sizes)
    X = (C[owner_of_row] + 0.8 * rng.standard_normal((len(owner_of_row), d))).astype(np.float32)
    Q = (C[rng.integers(0, L, nq)] + 0.8 * rng.standard_normal((nq, d))).astype(np.float32)
    ids = np.arange(len(X), dtype=np.int64) * 3 + 1
    alive = (rng.random(len(X)) > 0.05).astype(np.uint8)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    return dict(C=C, X=X, Q=Q, ids=ids, alive=alive, off=off, sizes=sizes, k=k, nprobe=nprobe)


def _local_lists(O, c, owner, rank):
    """CSR lists of this rank: its own lists' rows, the others empty."""
    off, X, ids, alive = c["off"], c["X"], c["ids"], c["alive"]
    keep = np.concatenate([np.arange(off[l], off[l + 1]) for l in range(len(off) - 1)
                           if owner[l] == rank] + [np.zeros(0, np.int64)]).astype(np.int64)
    lens = np.array([off[l + 1] - off[l] if owner[l] == rank else 0
                     for l in range(len(off) - 1)], np.int64)
    loff = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    return O.CsrLists(loff, X[keep], ids[keep], alive[keep])


def _rank_main(rank, world, port, metric, normalized, out):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from m3_memory_b200.sharding import shard_lists
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        c = _case()
        owner = shard_lists(c["sizes"], world)
        lists = _local_lists(O, c, owner, rank)
        ids, sc, cnt = O.search_nprobe(c["Q"], c["C"], lists, metric, normalized, c["k"],
                                       c["nprobe"])
        g_sc = [torch.empty_like(torch.from_numpy(sc)) for _ in range(world)]
        g_ids = [torch.empty_like(torch.from_numpy(ids)) for _ in range(world)]
        dist.all_gather(g_sc, torch.from_numpy(sc))
        dist.all_gather(g_ids, torch.from_numpy(ids))
        if rank == 0:
            merged = O.merge_shards(np.stack([t.numpy() for t in g_sc]),
                                    np.stack([t.numpy() for t in g_ids]))
            out.put(("ok", merged, owner))
    except Exception as ex:  # reported to the parent, which fails the test
        out.put(("error", repr(ex), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("metric,normalized", [(1, False), (0, False), (2, False)])
def test_sharded_search_equals_unsharded(oracle_mod, metric, normalized):
    from m3_memory_b200.sharding import shard_load, shard_lists

    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, metric, normalized, out))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        status, merged, owner = out.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert status == "ok", merged
    c = _case()
    np.testing.assert_array_equal(owner, shard_lists(c["sizes"], world))
    lists = oracle_mod.CsrLists(c["off"], c["X"], c["ids"], c["alive"])
    ref = oracle_mod.search_nprobe(c["Q"], c["C"], lists, metric, normalized, c["k"],
                                   c["nprobe"])
    compare_search(merged, ref, exact=True)
    assert all(p.exitcode == 0 for p in procs)
    # every list has one owner; the two ranks' rows differ by less than the largest list
    load = shard_load(c["sizes"], owner, world)
    assert load.sum() == c["sizes"].sum()
    assert abs(int(load[0]) - int(load[1])) <= int(c["sizes"].max())


def test_shard_lists_balance_and_determinism():
    from m3_memory_b200.sharding import shard_load, shard_lists

    rng = np.random.default_rng(0)
    sizes = rng.zipf(1.3, 4096) % 5000
    for world in (1, 2, 4, 8):
        owner = shard_lists(sizes, world)
        assert owner.min() >= 0 and owner.max() < world
        np.testing.assert_array_equal(owner, shard_lists(sizes.copy(), world))
        load = shard_load(sizes, owner, world)
        assert load.sum() == sizes.sum()
        assert load.max() - load.min() <= sizes.max()
    with pytest.raises(ValueError):
        shard_lists(sizes, 0)


def test_merge_shards_rule(oracle_mod):
    inf, nan = np.inf, np.nan
    sc = np.array([[[0.1, 0.3, inf]], [[0.1, 0.2, nan]]], np.float32)
    ids = np.array([[[5, 6, -1]], [[7, 8, -1]]], np.int64)
    got_ids, got_sc, cnt = oracle_mod.merge_shards(sc, ids)
    np.testing.assert_array_equal(got_ids, [[5, 7, 8]])  # tie 0.1: shard 0 first
    np.testing.assert_array_equal(got_sc, np.array([[0.1, 0.1, 0.2]], np.float32))
    np.testing.assert_array_equal(cnt, [3])


def test_global_top_p_from_ranks_exact_local_top_p(oracle_mod):
    """The sharded coarse step: every rank's exact top-P over its own centroids,
    merged by (exact score, rank, position), gives the single-index selection
    (all three metrics; the case has no exact score ties)."""
    from m3_memory_b200.sharding import shard_lists

    c = _case()
    L = len(c["C"])
    for world in (2, 3, 4):
        owner = shard_lists(c["sizes"], world)
        for metric, norm, P in ((1, False, 6), (0, False, 9), (2, False, 4)):
            sc = np.full((world, len(c["Q"]), P), np.inf, np.float32)
            ids = np.full((world, len(c["Q"]), P), -1, np.int64)
            for r in range(world):
                own = np.flatnonzero(owner == r)
                if len(own) == 0:
                    continue
                pl = min(P, len(own))
                for i, q in enumerate(c["Q"]):
                    loc = oracle_mod.select_nprobe(q, c["C"][own], metric, norm, pl)
                    sc[r, i, :pl] = [oracle_mod.score(q, c["C"][own[j]], metric, norm)
                                     for j in loc]
                    ids[r, i, :pl] = own[loc]
            top, _, cnt = oracle_mod.merge_shards(sc, ids)
            assert (cnt == min(P, L)).all()
            for i, q in enumerate(c["Q"]):
                want = oracle_mod.select_nprobe(q, c["C"], metric, norm, P)
                np.testing.assert_array_equal(top[i], want)


def _own_batch_rank_main(rank, world, port, metric, normalized, out):
    """The serving decomposition of ShardedSearch.search_own_batch with the oracle
    in place of the engine: every rank brings its own batch, the batches are
    all-gathered, each rank selects its own batch's probes, the probes are
    all-gathered, each rank searches its own lists for every query, and each
    batch's records go back to its rank through one all-to-all for the merge."""
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    from m3_memory_b200.sharding import shard_lists
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        c = _case()
        k, P = c["k"], c["nprobe"]
        B = len(c["Q"]) // world
        owner = shard_lists(c["sizes"], world)
        lists = _local_lists(O, c, owner, rank)
        q_own = torch.from_numpy(np.ascontiguousarray(c["Q"][rank * B:(rank + 1) * B]))
        q_all = torch.empty((world * B, q_own.shape[1]), dtype=torch.float32)
        dist.all_gather_into_tensor(q_all, q_own)
        loc = torch.from_numpy(np.stack([O.select_nprobe(q, c["C"], metric, normalized, P)
                                         for q in q_own.numpy()]).astype(np.int32))
        probes = torch.empty((world * B, P), dtype=torch.int32)
        dist.all_gather_into_tensor(probes, loc)
        ids = np.full((world * B, k), -1, np.int64)
        sc = np.full((world * B, k), np.inf, np.float32)
        for i, q in enumerate(q_all.numpy()):
            a_ids, a_sc, a_cnt = O.search_on(q[None], lists, probes[i].numpy(), metric,
                                             normalized, k)
            ids[i], sc[i] = a_ids[0], a_sc[0]
        # records of batch r (scores then ids, as bytes) go to rank r
        rec = [np.concatenate([sc[r * B:(r + 1) * B].reshape(-1).view(np.uint8),
                               ids[r * B:(r + 1) * B].reshape(-1).view(np.uint8)])
               for r in range(world)]
        send = torch.from_numpy(np.concatenate(rec))
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send)
        R = len(rec[0])
        got = recv.numpy().reshape(world, R)
        g_sc = got[:, :B * k * 4].copy().view(np.float32).reshape(world, B, k)
        g_ids = got[:, B * k * 4:].copy().view(np.int64).reshape(world, B, k)
        out.put((rank, "ok", O.merge_shards(g_sc, g_ids)))
    except Exception as ex:  # reported to the parent, which fails the test
        out.put((rank, "error", repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("metric,normalized", [(1, False), (0, False)])
def test_own_batch_exchange_equals_unsharded(oracle_mod, metric, normalized):
    """Each rank's merged answer for its own batch equals the unsharded search of
    that batch (world size 2 over gloo)."""
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_own_batch_rank_main,
                         args=(r, world, port, metric, normalized, out)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = [out.get(timeout=120) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    c = _case()
    B = len(c["Q"]) // world
    lists = oracle_mod.CsrLists(c["off"], c["X"], c["ids"], c["alive"])
    for rank, status, merged in res:
        assert status == "ok", merged
        want = oracle_mod.search_nprobe(c["Q"][rank * B:(rank + 1) * B], c["C"], lists, metric,
                                        normalized, c["k"], c["nprobe"])
        compare_search(merged, want, exact=True)
    assert all(p.exitcode == 0 for p in procs)


def _limit_rank_main(rank, world, port, mode, out):
    """Rank 0 runs one exchange with a 2 s host-side limit; rank 1 joins
    ("join"), leaves the job before it ("exit"), or stays but never joins
    ("stall")."""
    sys.path.insert(0, str(ROOT))
    import time

    import torch
    import torch.distributed as dist

    from m3_memory_b200.sharding import PendingCollective, ShardError, collective

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=6))
    src = torch.full((4,), float(rank + 1))
    dst = torch.empty(4 * world)
    pending = mode.endswith("_pending")
    mode = mode.replace("_pending", "")
    if rank == 1 and mode == "exit":
        os._exit(0)  # leaves without joining and without a clean shutdown
    if rank == 1 and mode == "stall":
        time.sleep(12)
        os._exit(0)
    t0 = time.monotonic()
    try:
        if pending:  # issued first, waited for after other work
            work = PendingCollective(dist.all_gather_into_tensor, 2.0, "probe exchange", dst, src)
            time.sleep(0.1)
            work.finish()
        else:
            collective(dist.all_gather_into_tensor, 2.0, "probe exchange", dst, src)
        res = ("ok", dst.tolist(), time.monotonic() - t0)
    except ShardError as ex:
        res = ("shard_error", str(ex), time.monotonic() - t0)
    except Exception as ex:  # anything else fails the test
        res = ("other", repr(ex), time.monotonic() - t0)
    if rank == 0:
        out.put(res)
        out.close()
        out.join_thread()  # the result is in the pipe before the process ends
    if res[0] == "ok":
        dist.destroy_process_group()
    os._exit(0)


@pytest.mark.parametrize("mode", ["join", "exit", "stall", "join_pending", "exit_pending"])
def test_exchange_limit_turns_a_missing_peer_into_an_error(mode):
    """The host-side limit on a sharded search's exchanges (ShardedSearch's
    timeout_s): with every rank present the exchange completes; a rank that left
    or never joins makes the waiting rank raise ShardError within the limit (or
    the process group's 6 s timeout), not block.  gloo ranks on CPU; no GPU."""
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_limit_rank_main, args=(r, world, port, mode, out))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        status, detail, elapsed = out.get(timeout=60)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    if mode.startswith("join"):
        assert status == "ok", detail
        assert detail == [1.0] * 4 + [2.0] * 4
    else:
        assert status == "shard_error", detail
        assert "probe exchange" in detail
        assert elapsed < 15, elapsed
