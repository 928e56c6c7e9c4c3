"""Search over the GPUs of one box with the inverted lists sharded by list.

Lists are independent units, so an index shards by list: every rank (one
process per GPU) keeps all centroids, so the coarse selection is replicated
and identical on every rank, loads only the lists it owns, and scans them for
the whole query batch.  The per-rank top-k answers ``[Q, k]`` (scores and ids)
go through one all-gather (NCCL over NVLink) and are merged on the GPU by
``m3g_merge_shards_device``: the k smallest by (score, rank, position), which
is the final ascending sort of ``IVFIndex::search_nprobe``
(AgentMemory/M3/src/m3_index.cpp:444-475) applied across shards.

The exchange is the only collective on the path; its size is
``world * Q * k * 12`` bytes per batch.
"""
from __future__ import annotations

import numpy as np


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
    ``max_q`` queries.
    """

    def __init__(self, engine, index_id: int, k: int, max_q: int, world: int, device,
                 group=None):
        import torch

        self.engine, self.index_id, self.k, self.world = engine, index_id, k, world
        self.group = group
        self.ids = torch.empty((max_q, k), dtype=torch.int64, device=device)
        self.sc = torch.empty((max_q, k), dtype=torch.float32, device=device)
        self.cnt = torch.empty((max_q,), dtype=torch.int32, device=device)
        self.g_ids = torch.empty((world, max_q, k), dtype=torch.int64, device=device)
        self.g_sc = torch.empty((world, max_q, k), dtype=torch.float32, device=device)
        self.out_ids = torch.empty((max_q, k), dtype=torch.int64, device=device)
        self.out_sc = torch.empty((max_q, k), dtype=torch.float32, device=device)
        self.out_cnt = torch.empty((max_q,), dtype=torch.int32, device=device)
        self.max_q = max_q

    def search(self, q, nprobe: int):
        """Top-k over all shards for the device query batch ``q`` ([nq, dim]
        fp32, nq <= max_q), enqueued on torch's current stream (the collectives
        are ordered after it).  Returns (ids, scores, counts) views of device
        buffers that the next call overwrites."""
        import torch
        import torch.distributed as dist

        nq = int(q.shape[0])
        if nq > self.max_q:
            raise ValueError(f"batch of {nq} queries exceeds max_q={self.max_q}")
        k = self.k
        s = torch.cuda.current_stream(q.device).cuda_stream
        self.engine.search_device(self.index_id, q.data_ptr(), nq, k, nprobe,
                                  self.ids.data_ptr(), self.sc.data_ptr(), self.cnt.data_ptr(), s)
        if self.world == 1:
            return self.ids[:nq], self.sc[:nq], self.cnt[:nq]
        # [world, nq, k] views over the start of the gather buffers (contiguous)
        g_sc = self.g_sc.view(-1)[:self.world * nq * k].view(self.world, nq, k)
        g_ids = self.g_ids.view(-1)[:self.world * nq * k].view(self.world, nq, k)
        dist.all_gather_into_tensor(g_sc, self.sc[:nq], group=self.group)
        dist.all_gather_into_tensor(g_ids, self.ids[:nq], group=self.group)
        self.engine.merge_shards_device(g_sc.data_ptr(), g_ids.data_ptr(), self.world, nq, k,
                                        self.out_ids.data_ptr(), self.out_sc.data_ptr(),
                                        self.out_cnt.data_ptr(), s)
        return self.out_ids[:nq], self.out_sc[:nq], self.out_cnt[:nq]
