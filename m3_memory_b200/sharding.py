"""Search over the GPUs of one box with the inverted lists sharded by list.

Lists are independent units, so an index shards by list: every rank (one
process per GPU) keeps all centroids, so the coarse selection is replicated
and identical on every rank, loads only the lists it owns, and scans them for
the whole query batch.  The per-rank top-k answers ``[Q, k]`` (scores and ids)
go through one all-gather (NCCL over NVLink) and are merged on the GPU by
``m3g_merge_shards_device``: the k smallest by (score, rank, position), which
is the final ascending sort of ``IVFIndex::search_nprobe``
(AgentMemory/M3/src/m3_index.cpp:444-475) applied across shards.

The exchange is the only collective on the path: each rank's answer is one
record (its ``[Q, k]`` fp32 scores, then its ``[Q, k]`` int64 ids), so a single
all-gather of ``world * Q * k * 12`` bytes per batch moves both, and the merge
reads the gathered records in place (``m3g_merge_shards_packed_device``).

With ``split_coarse=True`` the coarse step is split by query instead of being
repeated: rank r selects the probes of its slice of the batch (queries
r * ceil(Q / world) ..) over all centroids (``m3g_select_probe_sets_device``: the
same exact selection, each row's order left to the engine), the ``[Q, P]`` probe
lists are all-gathered (Q * P * 4
bytes), and every rank scans its own lists for the whole batch
(``m3g_search_probes_device``; lists it does not own hold no rows here) before
the top-k exchange above.  The coarse work per rank then shrinks with the
number of GPUs.

With ``coarse_index_id`` the coarse step is sharded too, so it shrinks with the
number of GPUs instead of being repeated on each: every rank keeps a second
index holding only the centroids of its own lists (ascending cluster id), takes
their exact top-P (``m3g_select_probes_device``) with exact scores
(``m3g_probe_scores_device``, the reference's arithmetic), the ``[Q, P]``
candidates of all ranks are all-gathered and merged into the global top-P by
(score, rank, position) -- the same P lists, in the same order, as the
single-GPU selection except between centroids whose exact scores tie -- and each
rank scans the winners it owns (``m3g_search_probes_device``, -1 for the
others) before the top-k exchange above.

``search_own_batch`` is the serving form, where every rank brings its own batch
of queries per step: the batches are all-gathered so that every shard sees
every query, each rank selects the probes of its own batch, the probe lists
are all-gathered, each rank scans its lists for all batches, and each batch's
per-shard top-k go back to the batch's rank in one all-to-all of packed records
for the final merge there.  The work per rank then stays fixed as ranks (and
batches) are added.
"""
from __future__ import annotations

import datetime

import numpy as np


class ShardError(RuntimeError):
    """An exchange of a sharded search did not complete: a peer rank left, failed
    or did not join within the limit.  The reference has no multi-GPU path; its
    writer-thread failures end the process (AgentMemory/M3/src/m3_async.cpp:364)."""


def collective(op, timeout_s, what, *args, **kwargs):
    """Runs one torch.distributed collective.  Without a limit it is enqueued as
    usual (ordered on the current stream, the host does not wait).  With
    timeout_s the host waits for it, at most that long, and a peer that does not
    join (or a transport error) raises ShardError naming the exchange instead of
    blocking the rank -- the host-side limit on every exchange of the search."""
    if timeout_s is None:
        return op(*args, **kwargs)
    try:
        work = op(*args, async_op=True, **kwargs)
        done = work.wait(timeout=datetime.timedelta(seconds=timeout_s))
    except Exception as ex:  # noqa: BLE001 -- every transport error becomes a ShardError
        raise ShardError(f"{what}: the exchange did not complete within {timeout_s} s "
                         f"({type(ex).__name__}: {ex})") from ex
    if done is False:
        raise ShardError(f"{what}: the exchange did not complete within {timeout_s} s")
    return None


class PendingCollective:
    """A collective issued now and waited for later, so that independent work can
    run between: without a limit, finish() makes the current stream wait for it;
    with timeout_s, finish() waits on the host, at most that long (ShardError)."""

    def __init__(self, op, timeout_s, what, *args, **kwargs):
        self.timeout_s, self.what = timeout_s, what
        try:
            self.work = op(*args, async_op=True, **kwargs)
        except Exception as ex:  # noqa: BLE001 -- transport errors become ShardErrors
            raise ShardError(f"{what}: the exchange could not start ({type(ex).__name__}: "
                             f"{ex})") from ex

    def finish(self):
        try:
            if self.timeout_s is None:
                self.work.wait()
                return
            done = self.work.wait(timeout=datetime.timedelta(seconds=self.timeout_s))
        except Exception as ex:  # noqa: BLE001
            raise ShardError(f"{self.what}: the exchange did not complete within "
                             f"{self.timeout_s} s ({type(ex).__name__}: {ex})") from ex
        if done is False:
            raise ShardError(f"{self.what}: the exchange did not complete within "
                             f"{self.timeout_s} s")


def torch_dtype(name):
    import torch

    return getattr(torch, name)


def shard_lists(sizes, world: int) -> np.ndarray:
    """Owner rank of every list: largest list first onto the least-loaded rank
    (ties: lower list id first, lower rank first), the same on every rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    sizes = np.asarray(sizes, dtype=np.int64)
    load = np.zeros(world, dtype=np.int64)
    owner = np.empty(len(sizes), np.int32)
    for lst in np.argsort(-sizes, kind="stable"):
        r = int(np.argmin(load))
        owner[lst] = r
        load[r] += int(sizes[lst])
    return owner


def shard_load(sizes, owner, world: int) -> np.ndarray:
    """Rows owned by each rank."""
    return np.bincount(np.asarray(owner), weights=np.asarray(sizes, dtype=np.float64),
                       minlength=world).astype(np.int64)


class ShardedSearch:
    """The per-batch exchange of a list-sharded search on one rank.

    ``engine`` is the rank's ``cabi.Engine`` holding all centroids and the
    lists this rank owns; ``group`` a ``torch.distributed`` process group over
    the ranks (NCCL on GPUs).  Buffers are allocated once for batches of up to
    ``max_q`` queries.  With ``timeout_s`` the host waits for every exchange, at
    most that long, and raises ``ShardError`` when a peer left, failed or did not
    join (without it the exchanges are only enqueued, and a missing peer holds the
    rank until the process group's own timeout).
    """

    def __init__(self, engine, index_id: int, k: int, max_q: int, world: int, device,
                 group=None, coarse_index_id=None, owner=None, rank: int = 0,
                 max_nprobe: int = 256, split_coarse: bool = False,
                 timeout_s: float | None = None):
        import torch

        self.engine, self.index_id, self.k, self.world = engine, index_id, k, world
        self.group = group
        # host-side limit on every exchange (None: enqueue and do not wait)
        self.timeout_s = timeout_s
        self.coarse_index_id = coarse_index_id
        self.split_coarse = split_coarse and coarse_index_id is None
        self.rank = rank
        self.max_probe_cap = max_nprobe
        if self.split_coarse:
            self.nlist = int(engine.info(index_id)[3])
            p = min(max_nprobe, self.nlist)
            chunk = -(-max_q // world)
            self.sp_loc = torch.empty((chunk, p), dtype=torch.int32, device=device)
            self.sp_all = torch.empty((world * chunk, p), dtype=torch.int32, device=device)
            self.max_nprobe = p
        if coarse_index_id is not None:
            if owner is None:
                raise ValueError("a sharded coarse step needs the list owners")
            owner = np.asarray(owner, dtype=np.int32)
            own = np.flatnonzero(owner == rank).astype(np.int64)
            self.nlist = len(owner)
            self.n_own = len(own)
            self.own_ids = torch.from_numpy(own).to(device)          # local -> global id
            self.owner = torch.from_numpy(owner).to(device)
            self.rank = rank
            p = min(max_nprobe, self.nlist)
            self.loc = torch.empty((max_q, p), dtype=torch.int32, device=device)
            self.loc_sc = torch.empty((max_q, p), dtype=torch.float32, device=device)
            self.cand_sc = torch.empty((max_q, p), dtype=torch.float32, device=device)
            self.cand_id = torch.empty((max_q, p), dtype=torch.int64, device=device)
            self.gc_sc = torch.empty((world, max_q, p), dtype=torch.float32, device=device)
            self.gc_id = torch.empty((world, max_q, p), dtype=torch.int64, device=device)
            self.top_id = torch.empty((max_q, p), dtype=torch.int64, device=device)
            self.top_sc = torch.empty((max_q, p), dtype=torch.float32, device=device)
            self.top_cnt = torch.empty((max_q,), dtype=torch.int32, device=device)
            self.max_nprobe = p
        self.ids = torch.empty((max_q, k), dtype=torch.int64, device=device)
        self.sc = torch.empty((max_q, k), dtype=torch.float32, device=device)
        self.cnt = torch.empty((max_q,), dtype=torch.int32, device=device)
        # this rank's answer as one record (scores, then ids), and the gathered records
        self.rec = torch.empty(self.record_bytes(max_q), dtype=torch.uint8, device=device)
        self.g_rec = torch.empty(world * self.record_bytes(max_q), dtype=torch.uint8,
                                 device=device)
        self.out_ids = torch.empty((max_q, k), dtype=torch.int64, device=device)
        self.out_sc = torch.empty((max_q, k), dtype=torch.float32, device=device)
        self.out_cnt = torch.empty((max_q,), dtype=torch.int32, device=device)
        self.max_q = max_q
        # every engine call and collective of a search runs on this one stream, so the
        # engine's kernels and NCCL's writes are ordered with each other; it waits for
        # the caller's stream on entry and the caller's stream waits for it on exit
        self.stream = torch.cuda.Stream(device)
        # set to a list to have search() append (phase, CUDA event) pairs, recorded on
        # the search's stream at the end of each phase ("start" first)
        self.marks = None

    def record_bytes(self, nq: int) -> int:
        """Bytes of one rank's answer record for nq queries: [nq, k] fp32 scores,
        padded to 8 bytes, then [nq, k] int64 ids."""
        return self.ids_offset(nq) + nq * self.k * 8

    def ids_offset(self, nq: int) -> int:
        return (nq * self.k * 4 + 7) // 8 * 8

    def _answer_views(self, nq):
        """Where this rank's search writes its answer: for world > 1 straight into
        its record (scores, ids), else the plain buffers."""
        if self.world == 1:
            return self.ids[:nq], self.sc[:nq]
        k, off = self.k, self.ids_offset(nq)
        sc = self.rec[:nq * k * 4].view(torch_dtype("float32")).view(nq, k)
        ids = self.rec[off:off + nq * k * 8].view(torch_dtype("int64")).view(nq, k)
        return ids, sc

    def _mark(self, name):
        if self.marks is not None:
            import torch

            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))

    def search(self, q, nprobe: int):
        """Top-k over all shards for the device query batch ``q`` ([nq, dim]
        fp32, nq <= max_q), ordered after torch's current stream, which waits for
        the answer.  Returns (ids, scores, counts) views of device buffers that the
        next call overwrites."""
        import torch

        caller = torch.cuda.current_stream(q.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            out = self._search(q, nprobe)
        caller.wait_stream(self.stream)
        return out

    def _search(self, q, nprobe: int):
        import torch
        import torch.distributed as dist

        nq = int(q.shape[0])
        if nq > self.max_q:
            raise ValueError(f"batch of {nq} queries exceeds max_q={self.max_q}")
        k = self.k
        s = self.stream.cuda_stream
        self._mark("start")
        a_ids, a_sc = self._answer_views(nq)
        if self.coarse_index_id is not None:
            self._search_sharded_coarse(q, nq, nprobe, s, a_ids, a_sc)
        elif self.split_coarse:
            self._search_split_coarse(q, nq, nprobe, s, a_ids, a_sc)
        else:
            self.engine.search_device(self.index_id, q.data_ptr(), nq, k, nprobe,
                                      a_ids.data_ptr(), a_sc.data_ptr(), self.cnt.data_ptr(), s)
            self._mark("search")
        if self.world == 1:
            return self.ids[:nq], self.sc[:nq], self.cnt[:nq]
        # one all-gather of the answer records, merged where they land
        R = self.record_bytes(nq)
        g = self.g_rec[:self.world * R]
        collective(dist.all_gather_into_tensor, self.timeout_s, "top-k exchange", g,
                   self.rec[:R], group=self.group)
        self.engine.merge_shards_packed_device(g.data_ptr(), self.world, nq, k, R,
                                               self.ids_offset(nq), self.out_ids.data_ptr(),
                                               self.out_sc.data_ptr(), self.out_cnt.data_ptr(), s)
        self._mark("topk_exchange")
        return self.out_ids[:nq], self.out_sc[:nq], self.out_cnt[:nq]

    def search_own_batch(self, q_own, nprobe: int):
        """Top-k over all shards for this rank's own query batch ``q_own`` ([B, dim]
        fp32, B <= max_q and the same on every rank), ordered after torch's current
        stream, which waits for the answer.

        Every rank brings its own batch per step: the batches are all-gathered
        (the queries reach every shard), each rank selects the probes of its own
        batch over all centroids, the probe lists are all-gathered, every rank
        scans its own lists for all world * B queries, and the per-shard top-k of
        each batch go back to the batch's rank -- one all-to-all of packed records
        (scores, then ids) -- where ``m3g_merge_shards_packed_device`` merges them.
        Per-rank work stays fixed as ranks are added.  Returns (ids, scores,
        counts) views of this rank's answer, overwritten by the next call."""
        import torch

        caller = torch.cuda.current_stream(q_own.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            out = self._search_own_batch(q_own, nprobe)
        caller.wait_stream(self.stream)
        return out

    def _own_buffers(self, dim, device):
        import torch

        if getattr(self, "_own", None) is not None and self._own["dim"] == dim:
            return self._own
        nlist = int(self.engine.info(self.index_id)[3])
        p = min(self.max_probe_cap, nlist)
        W, B, k = self.world, self.max_q, self.k
        R = self.record_bytes(B)
        self._own = dict(
            dim=dim, nlist=nlist, P=p,
            q_all=torch.empty((W * B, dim), dtype=torch.float32, device=device),
            loc=torch.empty((B, p), dtype=torch.int32, device=device),
            probes=torch.empty((W * B, p), dtype=torch.int32, device=device),
            ids=torch.empty((W * B, k), dtype=torch.int64, device=device),
            sc=torch.empty((W * B, k), dtype=torch.float32, device=device),
            cnt=torch.empty((W * B,), dtype=torch.int32, device=device),
            send=torch.empty(W * R, dtype=torch.uint8, device=device),
            recv=torch.empty(W * R, dtype=torch.uint8, device=device))
        return self._own

    def _search_own_batch(self, q, nprobe: int):
        import torch
        import torch.distributed as dist

        B, dim = int(q.shape[0]), int(q.shape[1])
        if B > self.max_q:
            raise ValueError(f"batch of {B} queries exceeds max_q={self.max_q}")
        if not q.is_contiguous():
            raise ValueError("the query batch must be contiguous")
        k, W, s = self.k, self.world, self.stream.cuda_stream
        self._mark("start")
        if W == 1:
            self.engine.search_device(self.index_id, q.data_ptr(), B, k, nprobe,
                                      self.ids.data_ptr(), self.sc.data_ptr(),
                                      self.cnt.data_ptr(), s)
            self._mark("search")
            return self.ids[:B], self.sc[:B], self.cnt[:B]
        o = self._own_buffers(dim, q.device)
        P = min(nprobe if nprobe > 0 else o["nlist"], o["nlist"])
        if P > o["P"]:
            raise ValueError(f"nprobe {P} exceeds max_nprobe={o['P']}")
        q_all = o["q_all"][:W * B]
        # the batches travel while this rank selects its own batch's probes (which
        # needs only its own queries); the scan waits for both
        gather = PendingCollective(dist.all_gather_into_tensor, self.timeout_s,
                                   "batch exchange", q_all, q, group=self.group)
        loc = o["loc"].view(-1)[:B * P].view(B, P)
        self.engine.select_probe_sets_device(self.index_id, q.data_ptr(), B, P, loc.data_ptr(),
                                             s)
        self._mark("coarse")
        gather.finish()
        self._mark("query_exchange")
        probes = o["probes"].view(-1)[:W * B * P].view(W * B, P)
        collective(dist.all_gather_into_tensor, self.timeout_s, "probe exchange", probes, loc,
                   group=self.group)
        self._mark("probe_exchange")
        ids, sc, cnt = o["ids"][:W * B], o["sc"][:W * B], o["cnt"][:W * B]
        self.engine.search_probes_device(self.index_id, q_all.data_ptr(), W * B, k,
                                         probes.data_ptr(), P, ids.data_ptr(), sc.data_ptr(),
                                         cnt.data_ptr(), s)
        self._mark("search")
        # batch r's answers from this shard go to rank r as one record
        R, off = self.record_bytes(B), self.ids_offset(B)
        send = o["send"][:W * R].view(W, R)
        send[:, :B * k * 4].view(torch.float32).copy_(sc.view(W, B * k))
        send[:, off:off + B * k * 8].view(torch.int64).copy_(ids.view(W, B * k))
        recv = o["recv"][:W * R]
        collective(dist.all_to_all_single, self.timeout_s, "top-k exchange", recv,
                   o["send"][:W * R], group=self.group)
        self.engine.merge_shards_packed_device(recv.data_ptr(), W, B, k, R, off,
                                               self.out_ids.data_ptr(), self.out_sc.data_ptr(),
                                               self.out_cnt.data_ptr(), s)
        self._mark("topk_exchange")
        return self.out_ids[:B], self.out_sc[:B], self.out_cnt[:B]

    def _search_split_coarse(self, q, nq, nprobe, s, a_ids, a_sc):
        """Probes of this rank's query slice, all-gathered, then the scan of the
        rank's lists for the whole batch; writes the rank's top-k to a_ids / a_sc
        (counts to self.cnt)."""
        import torch.distributed as dist

        P = min(nprobe if nprobe > 0 else self.nlist, self.nlist)
        if P > self.max_nprobe:
            raise ValueError(f"nprobe {P} exceeds max_nprobe={self.max_nprobe}")
        chunk = -(-nq // self.world)
        q0 = min(nq, self.rank * chunk)
        nloc = min(nq, q0 + chunk) - q0
        loc = self.sp_loc.view(-1)[:chunk * P].view(chunk, P)
        if nloc > 0:
            row = q.stride(0) * q.element_size()
            self.engine.select_probe_sets_device(self.index_id, q.data_ptr() + q0 * row, nloc,
                                                 P, loc.data_ptr(), s)
        if nloc < chunk:
            loc[nloc:].fill_(-1)
        self._mark("coarse")
        probes = self.sp_all.view(-1)[:self.world * chunk * P].view(self.world * chunk, P)
        if self.world > 1:
            collective(dist.all_gather_into_tensor, self.timeout_s, "probe exchange", probes, loc,
                       group=self.group)
        else:
            probes.copy_(loc)
        self._mark("probe_exchange")
        self.engine.search_probes_device(self.index_id, q.data_ptr(), nq, self.k,
                                         probes.data_ptr(), P, a_ids.data_ptr(),
                                         a_sc.data_ptr(), self.cnt.data_ptr(), s)
        self._mark("search")

    def _search_sharded_coarse(self, q, nq, nprobe, s, a_ids, a_sc):
        """Global top-P from the ranks' exact local top-P, then the scan of the
        winners this rank owns; writes the rank's top-k to a_ids / a_sc (counts to
        self.cnt)."""
        import torch
        import torch.distributed as dist

        P = min(nprobe if nprobe > 0 else self.nlist, self.nlist)
        if P > self.max_nprobe:
            raise ValueError(f"nprobe {P} exceeds max_nprobe={self.max_nprobe}")
        pl = min(P, self.n_own)
        cand_sc = self.cand_sc.view(-1)[:nq * P].view(nq, P)
        cand_id = self.cand_id.view(-1)[:nq * P].view(nq, P)
        cand_sc.fill_(float("inf"))
        cand_id.fill_(-1)
        if pl > 0:
            loc = self.loc.view(-1)[:nq * pl].view(nq, pl)
            loc_sc = self.loc_sc.view(-1)[:nq * pl].view(nq, pl)
            self.engine.select_probes_device(self.coarse_index_id, q.data_ptr(), nq, pl,
                                             loc.data_ptr(), s)
            self.engine.probe_scores_device(self.coarse_index_id, q.data_ptr(), nq,
                                            loc.data_ptr(), pl, loc_sc.data_ptr(), s)
            cand_sc[:, :pl] = loc_sc
            cand_id[:, :pl] = self.own_ids[loc.long()]
        if self.world > 1:
            g_sc = self.gc_sc.view(-1)[:self.world * nq * P].view(self.world, nq, P)
            g_id = self.gc_id.view(-1)[:self.world * nq * P].view(self.world, nq, P)
            collective(dist.all_gather_into_tensor, self.timeout_s, "candidate exchange", g_sc,
                       cand_sc, group=self.group)
            collective(dist.all_gather_into_tensor, self.timeout_s, "candidate exchange", g_id,
                       cand_id, group=self.group)
        else:
            g_sc, g_id = cand_sc.unsqueeze(0), cand_id.unsqueeze(0)
        top_id = self.top_id.view(-1)[:nq * P].view(nq, P)
        top_sc = self.top_sc.view(-1)[:nq * P].view(nq, P)
        self.engine.merge_shards_device(g_sc.data_ptr(), g_id.data_ptr(), self.world, nq, P,
                                        top_id.data_ptr(), top_sc.data_ptr(),
                                        self.top_cnt.data_ptr(), s)
        mine = (top_id >= 0) & (self.owner[top_id.clamp(min=0)] == self.rank)
        probes = torch.where(mine, top_id, torch.full_like(top_id, -1)).to(torch.int32)
        self.engine.search_probes_device(self.index_id, q.data_ptr(), nq, self.k,
                                         probes.data_ptr(), P, a_ids.data_ptr(),
                                         a_sc.data_ptr(), self.cnt.data_ptr(), s)
