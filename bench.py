#!/usr/bin/env python
"""IVF search throughput on B200: QPS at recall@10 >= 0.95 (dim 1024) and the
list scan's HBM bandwidth.

Workload (one step = one search batch): 1M fp32 unit-norm vectors, dim 1024,
from a 1,000-component Gaussian mixture (component means N(0, I) normalised,
per-point noise sigma = 0.3 in norm, renormalised; seeded synthetic data, no
dataset), inner-product metric, nlist = 4096 lists by k-means (10 iterations,
seeded random init, exact assignment) on a seeded 262,144-row sample (64 rows
per list), then every row assigned to its nearest centroid; nprobe = 32,
k = 10, 10 batches of 1,024 queries from the same mixture, one batch per step.
Both arms build this same index (bit for bit: the k-means and the assignment
follow the reference's nearest_clusters rule exactly) and print its
fingerprint.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (under torchrun): the lists are partitioned over the ranks (largest
first onto the least-loaded rank); every rank holds all centroids, scans only
its own lists for the same query batch, the per-rank top-k go through one NCCL
all-gather, and the engine's merge kernel forms the answer.

--impl reference times the reference's own CPU implementation of the path
(IVFIndex::search_nprobe built from its sources, oracle/_ref) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_VEC = 1_000_000
DIM = 1024
NCOMP = 1000
SIGMA = 0.3
NLIST = 4096
NPROBE = 32
FIXED_NPROBE = False  # profiling cases: no recall sweep over nprobe
K = 10
BATCH = 1024
NBATCH = 10
KMEANS_ITERS = 10
KMEANS_SAMPLE = 262_144  # k-means training rows (64 per list), a seeded sample
SEED = 0
METRIC_IP = 1
WORKLOAD = (f"ivf-search: {N_VEC // 1_000_000}M x {DIM} fp32 unit-norm mixture({NCOMP}), "
            f"IP, nlist {NLIST}, nprobe {NPROBE}, k {K}, batch {BATCH}")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


_RESULT_OUT = None


def emit(obj):
    """The one JSON line on stdout (the result); everything else goes to stderr."""
    out = _RESULT_OUT or sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def keep_stdout_for_result():
    """Point file descriptor 1 at stderr for the rest of the process (libraries such as
    NCCL print banners there) and keep a private copy of the original stdout for the
    result line."""
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def kmeans_sample():
    """The seeded k-means training rows (ascending row order), the same in both arms."""
    m = min(N_VEC, KMEANS_SAMPLE)
    return np.sort(np.random.default_rng(SEED + 1).choice(N_VEC, m, replace=False))


def weak_mode(args, world):
    """N > 1 with every GPU bringing its own batch of queries per step (the
    default), as opposed to one batch split over the GPUs."""
    return world > 1 and args.scaling == "weak"


def bench_config(nprobe, world=1, weak=True):
    """The workload as both arms name it (identical by construction)."""
    return {"workload": WORKLOAD, "n_vectors": N_VEC, "dim": DIM, "nlist": NLIST,
            "nprobe": nprobe, "k": K, "batch": BATCH,
            "global_batch": BATCH * world if weak else BATCH,
            "metric": "inner product",
            "kmeans": (f"{KMEANS_ITERS} iterations, seeded random init, exact assignment, on a "
                       f"seeded {min(N_VEC, KMEANS_SAMPLE)}-row sample; every row then assigned "
                       "to its nearest centroid"),
            "l2_flush": "not needed: each step streams ~4 GB of lists (> 126 MB L2)"}


def index_fingerprint(C, assign):
    import hashlib

    h = hashlib.sha256(np.ascontiguousarray(C, np.float32).tobytes())
    h.update(np.ascontiguousarray(assign, np.int32).tobytes())
    return h.hexdigest()[:16]


def make_data():
    from m3_memory_b200 import synthetic as S

    rng = np.random.default_rng(SEED)
    if N_VEC != 1_000_000:
        log(f"note: reduced profiling case, {N_VEC} vectors / {NLIST} lists (not the headline)")
    means = S.mixture_means(NCOMP, DIM, rng)
    X, _ = S.gaussian_mixture(N_VEC, means, SIGMA, rng)
    Q, _ = S.gaussian_mixture(BATCH * NBATCH, means, SIGMA, rng)
    return X, Q.reshape(NBATCH, BATCH, DIM)


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: str):
        self.gpu = gpu
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.flush()

    def summary(self):
        rows = []
        try:
            for line in Path(self.f.name).read_text().splitlines():
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        finally:
            os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def gpu_selector(dev):
    import torch

    try:
        u = torch.cuda.get_device_properties(dev).uuid
        return "GPU-" + str(u)
    except Exception:
        return str(dev)


# ---------------------------------------------------------------- helpers
def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def scan_kernel_name():
    """The list-scan kernel the engine runs for this workload (inner product, k <= 32)."""
    return "list_scan_kernel" if os.environ.get("M3G_SCAN") == "simt" else "list_scan_tc_kernel"


def scan_traffic_per_launch():
    """dram bytes of one scan launch from the committed ncu summary, if any."""
    name = "list_scan_traffic.txt" if scan_kernel_name() == "list_scan_kernel" \
        else "list_scan_tc_traffic.txt"
    p = ROOT / "profiles" / name
    if p.is_file():
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                return int(line.split(":")[1])
    return None


def exact_topk_ip(X_dev, Q_dev, k):
    """Exact top-k by inner product (fp32 matmul, TF32 off), chunked over X."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    best_s = best_i = None
    step = 1 << 17
    for b in range(0, X_dev.shape[0], step):
        s = Q_dev @ X_dev[b:b + step].T
        v, i = torch.topk(s, k, dim=1)
        i = i + b
        if best_s is None:
            best_s, best_i = v, i
        else:
            cs, ci = torch.cat([best_s, v], 1), torch.cat([best_i, i], 1)
            best_s, o = torch.topk(cs, k, dim=1)
            best_i = torch.gather(ci, 1, o)
    return best_i


def recall_at_k(found_ids, exact_ids, k):
    hit = 0
    for a, b in zip(found_ids, exact_ids):
        hit += len(set(a[:k].tolist()) & set(b[:k].tolist()))
    return hit / (len(found_ids) * k)


def ref_index_of(C, X, assign):
    """The reference core's IVFIndex holding the given centroids and lists (rows of a
    list in ascending row order, ids = row numbers)."""
    from oracle import oracle as O

    ref = O.RefIndex(DIM, METRIC_IP, False)
    ref.set_centroids(C)
    order = np.argsort(assign, kind="stable")
    bounds = np.searchsorted(assign[order], np.arange(NLIST + 1))
    for c in range(NLIST):
        b, e = bounds[c], bounds[c + 1]
        if e > b:
            rows = order[b:e]
            ref.rebuild_cluster(c, rows.astype(np.int64), X[rows])
    return ref


def cpu_reference_qps(ref, Q_all, nprobe, threads, target_s=12.0):
    """The reference core's IVFIndex::search_nprobe on the host over a bounded sample
    of the queries: returns (qps, sample description, the queries' row numbers, the
    reference's answers (ids, scores, counts))."""
    Qf = Q_all.reshape(-1, DIM)
    probe = Qf[: max(threads, 1) * 2]
    t0 = time.perf_counter()
    ref.search_nprobe(probe, K, nprobe, threads=threads)
    rate = len(probe) / max(time.perf_counter() - t0, 1e-6)
    n = int(min(len(Qf), max(threads, rate * target_s)))
    t0 = time.perf_counter()
    ans = ref.search_nprobe(Qf[:n], K, nprobe, threads=threads)
    dt = time.perf_counter() - t0
    return (n / dt, f"{n} of the {len(Qf)} queries, search_nprobe split over {threads} threads",
            np.arange(n), ans)


def parity_vs_reference(got, want):
    """Our answers against the reference core's for the same queries on the same
    index: recall of its ids, the largest relative score difference over the ids
    both return, and how many queries' id lists are identical."""
    g_ids, g_sc, g_cnt = got
    r_ids, r_sc, r_cnt = want
    hit = tot = same = 0
    err = 0.0
    for q in range(len(r_cnt)):
        c = int(r_cnt[q])
        rmap = dict(zip(r_ids[q, :c].tolist(), r_sc[q, :c].tolist()))
        gi = g_ids[q, :int(g_cnt[q])].tolist()
        same += int(gi == r_ids[q, :c].tolist())
        for i, sc in zip(gi, g_sc[q, :len(gi)].tolist()):
            if i in rmap:
                hit += 1
                err = max(err, abs(sc - rmap[i]) / max(abs(rmap[i]), 1e-6))
        tot += c
    return {"recall_vs_reference": hit / max(tot, 1), "max_rel_score_err": err,
            "n_queries": int(len(r_cnt)), "identical_id_lists": same,
            "counts_equal": bool(np.array_equal(g_cnt, r_cnt)),
            "bar": "recall >= 0.999, relative score error <= 1e-3"}


def exact_topk_ip_host(X, Q, k, block=1 << 17):
    """Exact top-k ids by inner product on the host (fp32 BLAS), for the recall of
    the reference arm."""
    best_s = np.full((len(Q), k), -np.inf, np.float32)
    best_i = np.zeros((len(Q), k), np.int64)
    for b in range(0, len(X), block):
        s = Q @ X[b:b + block].T
        i = np.argpartition(-s, k - 1, axis=1)[:, :k]
        v = np.take_along_axis(s, i, 1)
        cs, ci = np.concatenate([best_s, v], 1), np.concatenate([best_i, i + b], 1)
        o = np.argpartition(-cs, k - 1, axis=1)[:, :k]
        best_s, best_i = np.take_along_axis(cs, o, 1), np.take_along_axis(ci, o, 1)
    return best_i


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O

    if not O.have_ref():
        try:
            O.build(ref=None)
        except Exception:
            pass
    if not O.have_ref():
        emit({"impl": "reference",
              "unavailable": "oracle/_ref/liboracle_ref.so (the reference core) "
                             "was not built on this box"})
        return
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    t_setup = time.perf_counter()
    X, Qb = make_data()
    # The same index as the GPU arm, built on the host without the GPU engine: the
    # same k-means (seeded init rows, exact nearest_clusters assignment, fp64
    # row-order means) with its E-steps proposed by host BLAS and settled in the
    # reference's own arithmetic wherever the BLAS bound leaves two candidates.
    C, _ = O.kmeans_train_fast(X[kmeans_sample()], NLIST, KMEANS_ITERS, SEED, METRIC_IP, False)
    assign = O.nearest_clusters_fast(X, C, METRIC_IP, False)
    ref = ref_index_of(C, X, assign)
    log(f"[reference] index built on the host in {time.perf_counter() - t_setup:.1f}s")
    nprobe = NPROBE
    found = []

    def one_step(i):
        ids, _, _ = ref.search_nprobe(Qb[i % NBATCH], K, nprobe, threads=threads)
        found.append((i % NBATCH, ids))

    for w in range(args.warmup):
        one_step(w)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one_step(i)
    dt = time.perf_counter() - t0
    qps = BATCH * args.steps / dt
    exact = exact_topk_ip_host(X, Qb[0], K)
    b0 = [ids for b, ids in found if b == 0][0]
    recall = recall_at_k(b0, exact, K)
    sample = f"{BATCH} queries (one full batch) per step over {threads} host threads"
    emit({
        "impl": "reference", "metric": "search QPS at recall@10>=0.95 (IVF, dim 1024)",
        "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak" if world == 1 or weak_mode(args, world) else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(nprobe, world, world == 1 or weak_mode(args, world)),
        "recall_at_10": recall,
        "index": {"fingerprint": index_fingerprint(C, assign),
                  "built": "host: BLAS-proposed exact k-means + assignment (setup, untimed)"},
        "parallelism": f"IVFIndex::search_nprobe, queries split over {threads} host threads",
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


# ---------------------------------------------------------------- our arm
def build_headline_index(eng, X, rank=0, world=1):
    """The headline index on the engine (index id 1): k-means on the seeded sample,
    every row assigned to its nearest centroid, this rank's lists loaded (ids = row
    numbers).  Returns (centroids, assignment, list owners)."""
    from m3_memory_b200.sharding import shard_lists

    t0 = time.perf_counter()
    C, _ = eng.kmeans(X[kmeans_sample()], NLIST, KMEANS_ITERS, SEED, METRIC_IP, False)
    eng.create_ivf(1, DIM, METRIC_IP, False, C)
    assign = eng.nearest_clusters(1, X)
    log(f"[rank {rank}] k-means {KMEANS_ITERS} it + assignment on the GPU: "
        f"{time.perf_counter() - t0:.1f}s")
    sizes = np.bincount(assign, minlength=NLIST)
    owner = shard_lists(sizes, world)
    order = np.argsort(assign, kind="stable")
    bounds = np.searchsorted(assign[order], np.arange(NLIST + 1))
    for c in range(NLIST):
        b, e = bounds[c], bounds[c + 1]
        if e > b and owner[c] == rank:
            rows = order[b:e]
            eng.load_cluster(1, c, rows.astype(np.int64), X[rows])
    return C, assign, owner


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import ShardedSearch, shard_lists

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    t_setup = time.perf_counter()
    X, Qb = make_data()
    log(f"[rank {rank}] data ready in {time.perf_counter() - t_setup:.1f}s")
    eng = cabi.Engine()
    if args.tile_rows is not None:
        eng.set_scan_tile_rows(args.tile_rows)
    C, assign, owner = build_headline_index(eng, X, rank, world)
    log(f"[rank {rank}] index ready after {time.perf_counter() - t_setup:.1f}s")

    Qd = torch.from_numpy(Qb).to(dev)  # [NBATCH, BATCH, DIM]
    weak = weak_mode(args, world)
    coarse = {}
    if weak:
        coarse = dict(rank=rank)
    elif world > 1 and args.coarse == "split":
        coarse = dict(split_coarse=True, rank=rank)
    elif world > 1 and args.coarse == "sharded":
        # each rank scores only the centroids of the lists it owns
        eng.create_ivf(2, DIM, METRIC_IP, False, C[np.flatnonzero(owner == rank)])
        coarse = dict(coarse_index_id=2, owner=owner, rank=rank)
    sharded = ShardedSearch(eng, 1, K, BATCH, world, dev, **coarse)
    # queries answered per step by the whole job
    per_step = BATCH * world if weak else BATCH

    def own_batch(i):
        """The batch rank brings at step i (weak scaling: a different one per rank)."""
        return (i * world + rank) % NBATCH if weak else i % NBATCH

    def step(i, nprobe):
        if weak:
            ids, sc, _ = sharded.search_own_batch(Qd[own_batch(i)], nprobe)
        else:
            ids, sc, _ = sharded.search(Qd[i % NBATCH], nprobe)
        return ids, sc

    # ---- recall@10 against exact search (untimed); pick nprobe
    nprobe = NPROBE
    recall = None
    if rank == 0:
        Xd = torch.from_numpy(X).to(dev)
        exact = exact_topk_ip(Xd, Qd[0], K).cpu().numpy()
        del Xd
        torch.cuda.empty_cache()
    sweep = {}
    for p in (NPROBE,) if FIXED_NPROBE else (NPROBE, 48, 64, 96, 128, 256):
        found, _ = step(0, p)
        torch.cuda.synchronize()
        eng.sync_errors()
        r = recall_at_k(found.cpu().numpy(), exact, K) if rank == 0 else 0.0
        if world > 1:
            t = torch.tensor([r], device=dev)
            dist.broadcast(t, 0)
            r = float(t.item())
        sweep[p] = r
        if r >= 0.95 or FIXED_NPROBE:
            nprobe, recall = p, r
            break
    if recall is None:
        nprobe, recall = max(sweep, key=sweep.get), max(sweep.values())
    log(f"[rank {rank}] recall@10 sweep {sweep} -> nprobe {nprobe}")
    # every batch's answer at the chosen nprobe (untimed), for the parity check
    # against the reference core on the same index
    all_answers = [[], [], []]
    for b in range(NBATCH if world == 1 else 0):
        for lst, t in zip(all_answers, sharded.search(Qd[b], nprobe)):
            lst.append(t.cpu().numpy())

    # ---- device-resident timing
    for w in range(args.warmup):
        step(w, nprobe)
    torch.cuda.synchronize()
    eng.sync_errors()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_selector(local_rank)) as clk:
        torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" select this loop
        ev0.record()
        for i in range(args.steps):
            step(i, nprobe)
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    eng.sync_errors()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    qps = per_step * args.steps / (ms / 1e3)
    clocks = clk.summary()

    # ---- end to end through the C ABI with host buffers (H2D + D2H inside)
    pinned = torch.from_numpy(Qb).pin_memory()
    h_ids = torch.empty((BATCH, K), dtype=torch.int64).pin_memory()
    h_sc = torch.empty((BATCH, K), dtype=torch.float32).pin_memory()
    h_cnt = torch.empty((BATCH,), dtype=torch.int32).pin_memory()
    scan_ms, scan_bytes, launches = [], [], 0
    stage_ms = {}
    stage_by_rank = None  # N > 1: every rank's phase means
    if world == 1:
        lib = cabi.lib()

        def e2e_step(b):
            cabi.check(lib.m3g_search(eng.h, 1, pinned[b].data_ptr(), BATCH, K, nprobe,
                                      h_ids.data_ptr(), h_sc.data_ptr(), h_cnt.data_ptr()))

        for w in range(args.warmup):
            e2e_step(w % NBATCH)
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i % NBATCH)
        e2e_sync_s = time.perf_counter() - t0
        # the same steps with two in flight: step i uploads its batch (pinned host ->
        # device), searches it (m3g_search_device) and copies its answer back on stream
        # i % 2, so its upload overlaps step i - 1's search; the host reads step i's
        # answer (waits for its stream) before that slot is reused
        sl = [torch.cuda.Stream(dev) for _ in range(2)]
        qd = [torch.empty((BATCH, DIM), dtype=torch.float32, device=dev) for _ in range(2)]
        od = [(torch.empty((BATCH, K), dtype=torch.int64, device=dev),
               torch.empty((BATCH, K), dtype=torch.float32, device=dev),
               torch.empty((BATCH,), dtype=torch.int32, device=dev)) for _ in range(2)]
        hb = [(torch.empty((BATCH, K), dtype=torch.int64).pin_memory(),
               torch.empty((BATCH, K), dtype=torch.float32).pin_memory(),
               torch.empty((BATCH,), dtype=torch.int32).pin_memory()) for _ in range(2)]

        def launch(i):
            j = i % 2
            with torch.cuda.stream(sl[j]):
                qd[j].copy_(pinned[i % NBATCH], non_blocking=True)
                cabi.check(lib.m3g_search_device(eng.h, 1, qd[j].data_ptr(), BATCH, K, nprobe,
                                                 od[j][0].data_ptr(), od[j][1].data_ptr(),
                                                 od[j][2].data_ptr(), sl[j].cuda_stream))
                for h, o in zip(hb[j], od[j]):
                    h.copy_(o, non_blocking=True)

        def run_pipelined(n):
            for i in range(n):
                if i >= 2:
                    sl[i % 2].synchronize()  # step i - 2's answer is on the host
                launch(i)
            for x in sl:
                x.synchronize()

        run_pipelined(max(args.warmup, 2))
        eng.sync_errors()
        t0 = time.perf_counter()
        run_pipelined(args.steps)
        e2e_s = time.perf_counter() - t0
        eng.sync_errors()
        # per-stage device times, scan bytes and launch counts: the same calls again with
        # the engine's stage events on (outside the timed loops)
        eng.set_profiling(True)
        for i in range(args.steps):
            e2e_step(i % NBATCH)
            p = eng.last_profile()
            for key in ("ms_prep", "ms_coarse_gemm", "ms_select", "ms_worklist", "ms_scan",
                        "ms_merge", "ms_total"):
                stage_ms.setdefault(key, []).append(p[key])
            scan_ms.append(p["ms_scan"])
            scan_bytes.append(p["scan_bytes"])
            launches += p["kernel_launches"]
        eng.set_profiling(False)
    else:
        qdev = torch.empty((BATCH, DIM), dtype=torch.float32, device=dev)

        def e2e_step(i):
            qdev.copy_(pinned[own_batch(i)], non_blocking=True)
            if weak:
                m_ids, m_sc, m_cnt = sharded.search_own_batch(qdev, nprobe)
            else:
                m_ids, m_sc, m_cnt = sharded.search(qdev, nprobe)
            h_ids.copy_(m_ids, non_blocking=True)
            h_sc.copy_(m_sc, non_blocking=True)
            h_cnt.copy_(m_cnt, non_blocking=True)
            torch.cuda.synchronize()

        for w in range(args.warmup):
            e2e_step(w)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i)
        e2e_sync_s = time.perf_counter() - t0
        # the same steps with two in flight: step i uploads its batch, searches it (its
        # own ShardedSearch, stream and buffers; the engine orders the two on its
        # workspace) and copies the answer back on stream i % 2, so its upload and its
        # exchanges overlap step i - 1's work; every rank issues the same collectives
        # in the same order
        sl = [torch.cuda.Stream(dev) for _ in range(2)]
        ssl = [sharded, ShardedSearch(eng, 1, K, BATCH, world, dev, **coarse)]
        qd = [torch.empty((BATCH, DIM), dtype=torch.float32, device=dev) for _ in range(2)]
        hb = [(torch.empty((BATCH, K), dtype=torch.int64).pin_memory(),
               torch.empty((BATCH, K), dtype=torch.float32).pin_memory(),
               torch.empty((BATCH,), dtype=torch.int32).pin_memory()) for _ in range(2)]

        def launch(i):
            j = i % 2
            with torch.cuda.stream(sl[j]):
                qd[j].copy_(pinned[own_batch(i)], non_blocking=True)
                if weak:
                    out = ssl[j].search_own_batch(qd[j], nprobe)
                else:
                    out = ssl[j].search(qd[j], nprobe)
                for h, o in zip(hb[j], out):
                    h.copy_(o, non_blocking=True)

        def run_pipelined(n):
            for i in range(n):
                if i >= 2:
                    sl[i % 2].synchronize()  # step i - 2's answer is on the host
                launch(i)
            for x in sl:
                x.synchronize()

        run_pipelined(max(args.warmup, 2))
        dist.barrier()
        t0 = time.perf_counter()
        run_pipelined(args.steps)
        e2e_s = time.perf_counter() - t0
        t = torch.tensor([e2e_s, e2e_sync_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s, e2e_sync_s = float(t[0].item()), float(t[1].item())
        # per-phase device times of the device-resident step on this rank (every rank
        # runs the same calls; outside the timed loops)
        marks_per_step = []
        for i in range(min(args.steps, 50)):
            sharded.marks = []
            step(i, nprobe)
            marks_per_step.append(sharded.marks)
        sharded.marks = None
        torch.cuda.synchronize()
        for m in marks_per_step:
            for (_, ea), (name, eb) in zip(m, m[1:]):
                stage_ms.setdefault("ms_" + name, []).append(ea.elapsed_time(eb))
            stage_ms.setdefault("ms_total", []).append(m[0][1].elapsed_time(m[-1][1]))
        # every rank's phase means, gathered (the slowest rank's scan sets the step)
        names = sorted(stage_ms)
        mine = torch.tensor([statistics.mean(stage_ms[k]) for k in names], device=dev)
        every = torch.empty((world, len(names)), device=dev)
        dist.all_gather_into_tensor(every, mine)
        stage_by_rank = {k[3:]: [round(float(x), 4) for x in every[:, j].tolist()]
                         for j, k in enumerate(names)}
    e2e_qps = per_step * args.steps / e2e_s
    e2e_sync_qps = per_step * args.steps / e2e_sync_s

    if rank != 0:
        return
    # our kernels per step: query prep (norms + split), coarse GEMM, select, 5 work-list
    # (histogram, gather, scan, place, pair scatter), scan, merge; N > 1 adds the shard
    # merge; the query-split coarse step a second prep and the partial-list clear; the
    # sharded coarse step also the pair scores and the top-P merge; the own-batch (weak)
    # step: prep, coarse GEMM, select for the rank's batch, then prep, 5 work-list,
    # partial clear, scan, merge for all batches, and the shard merge
    # (the profiled calls add the engine's probed-byte counter, one launch per step, which
    # the timed loop does not run)
    per_step_launches = (launches / args.steps - 1) if launches else (
        10 if world == 1 else 13 if weak else
        {"replicated": 11, "split": 13, "sharded": 15}[args.coarse])
    peak, peak_kind = peaks()
    roofline = None
    if scan_ms:
        avg_ms = statistics.mean(scan_ms)
        avg_bytes = statistics.mean(scan_bytes)
        achieved = avg_bytes / (avg_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": scan_traffic_per_launch(),
                    "kernel": scan_kernel_name(),
                    "bytes_per_launch": avg_bytes, "ms_per_launch": avg_ms,
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                    if peak_kind == "measured" else "fallback 6650 GB/s"}
    cpu = parity = None
    if world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O

        if O.have_ref():
            threads = len(os.sched_getaffinity(0))
            ref = ref_index_of(C, X, assign)
            v, sample, qrows, want = cpu_reference_qps(ref, Qb, nprobe, threads)
            del ref
            cpu = {"value": v, "unit": "queries/s", "cores": threads, "kind": "reference",
                   "sample": sample}
            got = tuple(np.concatenate([a[i] for i in range(NBATCH)])[qrows]
                        for a in all_answers)
            parity = parity_vs_reference(got, want)
    line = {
        "metric": "search QPS at recall@10>=0.95 (IVF, dim 1024)",
        "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 and not weak else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture; no dataset)",
        "config": bench_config(nprobe, world, world == 1 or weak),
        "recall_at_10": recall,
        "recall_sweep": {str(k): v for k, v in sweep.items()},
        "stage_ms_mean": {k[3:]: round(statistics.mean(v), 4) for k, v in stage_ms.items()},
        "stage_ms_by_rank": stage_by_rank,
        "parallelism": ("1 GPU" if world == 1 else
                        f"lists sharded over {world} GPUs; every GPU brings its own batch of "
                        f"{BATCH} queries per step (batches all-gathered, probes of each batch "
                        "selected on its GPU and all-gathered, per-shard top-k returned to the "
                        "batch's GPU by one all-to-all)" if weak else
                        f"lists sharded over {world} GPUs, one batch per step, {args.coarse} "
                        "coarse selection"),
        "index": {"fingerprint": index_fingerprint(C, assign),
                  "built": "GPU: m3g_kmeans on the sample + m3g_nearest_clusters (setup, untimed)"},
        "parity": parity,
        "gpu_launches": int(round(per_step_launches * args.steps)),
        "clocks": clocks,
        "e2e": {"value": e2e_qps, "unit": "queries/s",
                "h2d_bytes_per_step": BATCH * DIM * 4,
                "d2h_bytes_per_step": BATCH * K * 12 + BATCH * 4,
                "sync_call_value": e2e_sync_qps,
                "path": "pinned host queries -> H2D + m3g_search_device + D2H of the answer, two "
                        "steps in flight on alternating streams (sync_call_value: one blocking "
                        "m3g_search per step)" if world == 1
                else "per GPU: H2D of its own batch + NCCL all-gather of the batches + "
                     "m3g_select_probe_sets_device (own batch) + NCCL all-gather of the probes + "
                     "m3g_search_probes_device (all batches, own lists) + NCCL all-to-all of "
                     "the packed top-k records + m3g_merge_shards_packed_device + D2H of its "
                     "batch's answer, two steps in flight on alternating streams "
                     "(sync_call_value: one step at a time); bytes per GPU" if weak
                else ("H2D + m3g_search_device + NCCL all-gather + m3g_merge_shards_device + D2H"
                      if args.coarse == "replicated" else
                      "H2D + m3g_select_probe_sets_device (this rank's query slice) + NCCL all-gather "
                      "of the probes + m3g_search_probes_device + NCCL all-gather + "
                      "m3g_merge_shards_device + D2H" if args.coarse == "split" else
                      "H2D + m3g_select_probes_device + m3g_probe_scores_device (own centroids) + "
                      "NCCL all-gather + m3g_merge_shards_device (top-P) + "
                      "m3g_search_probes_device + NCCL all-gather + m3g_merge_shards_device + D2H")},
        "roofline": roofline,
        "cpu_baseline": cpu,
    }
    emit(line)


# ---------------------------------------------------------------- bf16-stored lists
# 10M x 768 vectors stored as bf16, 10k-component mixture, squared L2, nlist
# 16384, k 100, nprobe 8 / 32 / 128 and batches of 1 / 64 / 4096 queries.
C3_N = 10_000_000
C3_DIM = 768
C3_NCOMP = 10_000
C3_NLIST = 16384
C3_K = 100
C3_NPROBES = (8, 32, 128)
C3_BATCHES = (1, 64, 4096)
C3_NQ = 10_240
C3_SAMPLE_PER_LIST = 64


def device_mixture(n, nq, d, ncomp, sigma, seed, dev, chunk=1 << 20):
    """Seeded mixture data generated on the GPU (torch's CUDA generator), the
    same on every rank: unit-norm component means, points = mean + sigma / sqrt(d)
    noise, renormalised.  Returns (X [n, d] fp32, Q [nq, d] fp32) on dev."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    means = torch.randn(ncomp, d, generator=g, device=dev)
    means /= means.norm(dim=1, keepdim=True)

    def draw(m):
        out = torch.empty(m, d, device=dev)
        comp = torch.randint(0, ncomp, (m,), generator=g, device=dev)
        for b in range(0, m, chunk):
            e = min(m, b + chunk)
            x = means[comp[b:e]] + (sigma / d ** 0.5) * torch.randn(e - b, d, generator=g,
                                                                   device=dev)
            out[b:e] = x / x.norm(dim=1, keepdim=True)
        return out

    X = draw(n)
    Q = draw(nq)
    return X, Q


def exact_topk_l2_device(X, Q, k, step=1 << 20):
    """Exact top-k ids by squared L2 (fp32, TF32 off), chunked over X."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    best_s = best_i = None
    for b in range(0, X.shape[0], step):
        xb = X[b:b + step]
        s = 2.0 * (Q @ xb.T) - (xb * xb).sum(1)[None, :]  # larger is nearer
        v, i = torch.topk(s, k, dim=1)
        i = i + b
        if best_s is None:
            best_s, best_i = v, i
        else:
            cs, ci = torch.cat([best_s, v], 1), torch.cat([best_i, i], 1)
            best_s, o = torch.topk(cs, k, dim=1)
            best_i = torch.gather(ci, 1, o)
    return best_i


def run_config3(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import ShardedSearch, shard_lists

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n, d, nlist, K3 = args.c3_n or C3_N, C3_DIM, args.c3_nlist or C3_NLIST, args.c3_k or C3_K
    storage = cabi.BF16 if args.storage == "bf16" else cabi.F32
    t0 = time.perf_counter()
    X, Qd = device_mixture(n, C3_NQ, d, C3_NCOMP, SIGMA, SEED + 3, dev)
    log(f"[rank {rank}] {n} x {d} generated on the GPU in {time.perf_counter() - t0:.1f}s")
    eng = cabi.Engine()
    if args.tile_rows is not None:
        eng.set_scan_tile_rows(args.tile_rows)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 4)
    m = min(n, nlist * C3_SAMPLE_PER_LIST)
    sample = torch.randperm(n, generator=g, device=dev)[:m].sort().values
    t0 = time.perf_counter()
    C, _ = eng.kmeans(X[sample].cpu().numpy(), nlist, KMEANS_ITERS, SEED, 0, False)
    eng.create_ivf(1, d, 0, False, C, storage=storage)
    assign = torch.empty(n, dtype=torch.int32, device=dev)
    step = 1 << 21
    for b in range(0, n, step):
        e = min(n, b + step)
        eng.nearest_clusters_device(1, X[b:e].data_ptr(), e - b, assign[b:e].data_ptr())
    log(f"[rank {rank}] k-means ({KMEANS_ITERS} it on {m} rows) + assignment: "
        f"{time.perf_counter() - t0:.1f}s")
    sizes = torch.bincount(assign.long(), minlength=nlist).cpu().numpy()
    owner = shard_lists(sizes, world)
    t0 = time.perf_counter()
    # this rank's lists, loaded in one pass (rows of other ranks' lists: -1)
    own = torch.from_numpy(owner == rank).to(dev)
    mine = torch.where(own[assign.long()], assign, torch.full_like(assign, -1))
    row_ids = torch.arange(n, dtype=torch.int64, device=dev)
    eng.load_lists_device(1, mine.data_ptr(), row_ids.data_ptr(), X.data_ptr(), n)
    local_rows = int((mine >= 0).sum().item())
    del mine, row_ids
    torch.cuda.synchronize()
    log(f"[rank {rank}] {local_rows} rows loaded ({args.storage} lists) in "
        f"{time.perf_counter() - t0:.1f}s")
    exact = exact_topk_l2_device(X, Qd[:1024], 10).cpu().numpy() if rank == 0 else None
    del X, assign
    torch.cuda.empty_cache()

    sharded = ShardedSearch(eng, 1, K3, max(C3_BATCHES), world, dev, rank=rank,
                            max_nprobe=max(C3_NPROBES), split_coarse=world > 1)
    recall = {}
    for P in C3_NPROBES:
        ids, _, _ = sharded.search(Qd[:1024], P)
        torch.cuda.synchronize()
        r = recall_at_k(ids.cpu().numpy(), exact, 10) if rank == 0 else 0.0
        if world > 1:
            t = torch.tensor([r], device=dev)
            dist.broadcast(t, 0)
            r = float(t.item())
        recall[P] = r
    eng.sync_errors()
    ok = [P for P in C3_NPROBES if recall[P] >= 0.95]
    head_p = min(ok) if ok else max(recall, key=recall.get)
    log(f"[rank {rank}] recall@10 by nprobe {recall} -> headline nprobe {head_p}")

    def timed(P, B, steps):
        span = C3_NQ - B + 1
        for w in range(args.warmup):
            sharded.search(Qd[(w * B) % span:(w * B) % span + B], P)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(steps):
            o = (i * B) % span
            sharded.search(Qd[o:o + B], P)
        ev1.record()
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return B * steps / (ms / 1e3), ms / steps

    sweep = {}
    for P in C3_NPROBES:
        for B in C3_BATCHES:
            if (P, B) == (head_p, 4096):
                continue
            qps, ms = timed(P, B, min(args.steps, 50))
            sweep[f"nprobe{P}_batch{B}"] = {"qps": qps, "ms_per_step": ms, "recall_at_10": recall[P]}
    eng.sync_errors()
    with ClockSampler(gpu_selector(local_rank)) as clk:
        torch.cuda.nvtx.range_push("timed")  # ncu --nvtx-include "timed/" selects this loop
        qps, ms = timed(head_p, 4096, args.steps)
        torch.cuda.nvtx.range_pop()
    clocks = clk.summary()
    eng.sync_errors()
    sweep[f"nprobe{head_p}_batch4096"] = {"qps": qps, "ms_per_step": ms,
                                          "recall_at_10": recall[head_p]}
    if rank != 0:
        return
    # end to end, roofline, reference sample (one GPU only)
    e2e = roofline = cpu = parity = None
    B = 4096
    if world == 1:
        lib = cabi.lib()
        Qh = Qd.cpu().numpy()
        pinned = torch.from_numpy(Qh).pin_memory()
        h_ids = torch.empty((B, K3), dtype=torch.int64).pin_memory()
        h_sc = torch.empty((B, K3), dtype=torch.float32).pin_memory()
        h_cnt = torch.empty((B,), dtype=torch.int32).pin_memory()
        span = C3_NQ - B + 1

        def e2e_step(i):
            o = (i * B) % span
            cabi.check(lib.m3g_search(eng.h, 1, pinned[o].data_ptr(), B, K3, head_p,
                                      h_ids.data_ptr(), h_sc.data_ptr(), h_cnt.data_ptr()))

        for w in range(args.warmup):
            e2e_step(w)
        t0 = time.perf_counter()
        for i in range(args.steps):
            e2e_step(i)
        e2e = {"value": B * args.steps / (time.perf_counter() - t0), "unit": "queries/s",
               "h2d_bytes_per_step": B * d * 4, "d2h_bytes_per_step": B * K3 * 12 + B * 4,
               "path": "m3g_search (C ABI, pinned host buffers)"}
        eng.set_profiling(True)
        sm, sb, stages = [], [], {}
        for i in range(min(args.steps, 20)):
            e2e_step(i)
            p = eng.last_profile()
            sm.append(p["ms_scan"])
            sb.append(p["scan_bytes"])
            for key in ("ms_prep", "ms_coarse_gemm", "ms_select", "ms_worklist", "ms_scan",
                        "ms_merge", "ms_total"):
                stages.setdefault(key[3:], []).append(p[key])
        eng.set_profiling(False)
        peak, peak_kind = peaks()
        ach = statistics.mean(sb) / (statistics.mean(sm) / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                    "frac": ach / peak, "traffic": None, "kernel": "list_scan_tc_kernel<bf16 rows>",
                    "bytes_per_launch": statistics.mean(sb),
                    "ms_per_launch": statistics.mean(sm),
                    "stage_ms_mean": {k: round(statistics.mean(v), 4) for k, v in stages.items()},
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}
        # the stages of small batches (device-resident queries, the engine's events; the
        # kernels then run one by one instead of as a graph)
        small = {}
        ids_d = torch.empty((64, K3), dtype=torch.int64, device=dev)
        sc_d = torch.empty((64, K3), dtype=torch.float32, device=dev)
        cnt_d = torch.empty((64,), dtype=torch.int32, device=dev)
        eng.set_profiling(True)
        for Bs, Ps in ((1, C3_NPROBES[0]), (64, C3_NPROBES[0]), (1, C3_NPROBES[-1])):
            st_s = {}
            torch.cuda.nvtx.range_push(f"small{Bs}")  # ncu --nvtx-include "small1/" selects these
            for i in range(10):
                eng.search_device(1, Qd[i * Bs].data_ptr(), Bs, K3, Ps, ids_d.data_ptr(),
                                  sc_d.data_ptr(), cnt_d.data_ptr())
                p = eng.last_profile()
                for key in ("ms_prep", "ms_coarse_gemm", "ms_select", "ms_worklist", "ms_scan",
                            "ms_merge", "ms_total"):
                    st_s.setdefault(key[3:], []).append(p[key])
            torch.cuda.nvtx.range_pop()
            small[f"nprobe{Ps}_batch{Bs}"] = {
                k: round(statistics.median(v), 4) for k, v in st_s.items()}
        eng.set_profiling(False)
        roofline["small_batch_stage_ms_median"] = small
        if not args.no_cpu_baseline:
            from oracle import oracle as O

            if O.have_ref():
                nq_ref = 64
                Qs = Qh[:nq_ref]
                probes = eng.select_probes(1, Qs, head_p)
                need = np.unique(probes)
                ref = O.RefIndex(d, 0, False)
                ref.set_centroids(C)
                for c in need.tolist():
                    ci, cv = eng.get_cluster(1, c)  # the stored (bf16) values as fp32
                    if len(ci):
                        ref.rebuild_cluster(c, ci, cv)
                threads = len(os.sched_getaffinity(0))
                t0 = time.perf_counter()
                want = ref.search_nprobe(Qs, K3, head_p, threads=threads)
                v = nq_ref / (time.perf_counter() - t0)
                cpu = {"value": v, "unit": "queries/s", "cores": threads, "kind": "reference",
                       "sample": f"{nq_ref} queries, IVFIndex::search_nprobe over the lists "
                                 f"they probe ({len(need)} lists, stored values as fp32), "
                                 f"{threads} threads"}
                parity = parity_vs_reference(eng.search(1, Qs, K3, head_p), want)
    emit({
        "metric": "search QPS at recall@10>=0.95 (IVF, dim 768, bf16-stored lists)",
        "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16 rows, fp32 queries and accumulation",
        "data": "synthetic (seeded 10k-component Gaussian mixture generated on the GPU)",
        "config": {"workload": ("PROFILING CASE (not the bf16 configuration): "
                                if (args.c3_n or args.c3_k or args.c3_nlist) else "") +
                               f"ivf-search: {n // 1_000_000}M x {d} {args.storage}-stored "
                               f"mixture({C3_NCOMP}), L2, nlist {nlist}, nprobe {head_p}, "
                               f"k {K3}, batch {B}",
                   "n_vectors": n, "dim": d, "nlist": nlist, "nprobe": head_p, "k": K3,
                   "batch": B, "storage": args.storage, "metric": "squared L2",
                   "l2_flush": "not needed: each batch streams GBs of lists (> 126 MB L2)"},
        "recall_at_10": recall[head_p], "recall_by_nprobe": {str(k): v for k, v in recall.items()},
        "sweep": sweep,
        "parallelism": f"lists sharded over {world} GPU(s), split coarse selection"
        if world > 1 else "1 GPU",
        "gpu_launches": None, "clocks": clocks, "e2e": e2e, "roofline": roofline,
        "cpu_baseline": cpu, "parity": parity,
    })


# ---------------------------------------------------------------- Zipf-skewed shards
# Weak scaling by shard: every GPU holds one shard of 12.5M unit-norm rows x 1024
# (its own Zipf(1.1)-skewed mixture of 8192 components, k-means lists trained on
# the shard), the index is the union of the N shards (N x 8192 lists, every
# rank holding all centroids), cosine, nprobe 64, k 10, batches of 4096 x N
# queries drawn from the union.  At N = 8 this is the 100M x 1024, 65,536-list
# configuration.
C4_N = 12_500_000
C4_NLIST = 8192
C4_ZIPF = 1.1
C4_NPROBE = 64
C4_BATCH_PER_GPU = 4096


def device_zipf_means(ncomp, d, seed, dev):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    means = torch.randn(ncomp, d, generator=g, device=dev)
    return means / means.norm(dim=1, keepdim=True)


def device_zipf_rows(means, n, zipf, sigma, seed, dev, chunk=1 << 20):
    """n unit-norm rows of a mixture whose component c has weight ~ (c + 1)^-zipf."""
    import torch

    ncomp, d = means.shape
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.arange(1, ncomp + 1, device=dev, dtype=torch.float64) ** (-zipf)
    comp = torch.multinomial(w, n, replacement=True, generator=g)
    out = torch.empty(n, d, device=dev)
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        x = means[comp[b:e]] + (sigma / d ** 0.5) * torch.randn(e - b, d, generator=g, device=dev)
        out[b:e] = x / x.norm(dim=1, keepdim=True)
    return out


def run_config4(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from m3_memory_b200 import cabi
    from m3_memory_b200.sharding import ShardedSearch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n, d, nl = args.c4_n or C4_N, DIM, C4_NLIST
    B = C4_BATCH_PER_GPU * world
    t0 = time.perf_counter()
    means = [device_zipf_means(nl, d, SEED + 200 + r, dev) for r in range(world)]
    X = device_zipf_rows(means[rank], n, C4_ZIPF, SIGMA, SEED + 300 + rank, dev)
    eng = cabi.Engine()
    if args.tile_rows is not None:
        eng.set_scan_tile_rows(args.tile_rows)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 400 + rank)
    sample = torch.randperm(n, generator=g, device=dev)[:min(n, nl * 64)].sort().values
    C, _ = eng.kmeans(X[sample].cpu().numpy(), nl, KMEANS_ITERS, SEED + rank, 2, True)
    # the shard's own lists: every row to its nearest centroid of this shard
    eng.create_ivf(2, d, 2, True, C)
    assign = torch.empty(n, dtype=torch.int32, device=dev)
    for b in range(0, n, 1 << 21):
        e = min(n, b + (1 << 21))
        eng.nearest_clusters_device(2, X[b:e].data_ptr(), e - b, assign[b:e].data_ptr())
    # the union index: every shard's centroids (rank-major), this rank's lists
    Cd = torch.from_numpy(C).to(dev)
    if world > 1:
        Call = torch.empty((world * nl, d), device=dev)
        dist.all_gather_into_tensor(Call, Cd)
    else:
        Call = Cd
    eng.create_ivf(1, d, 2, True, Call.cpu().numpy())
    glob = assign + rank * nl
    row_ids = torch.arange(n, dtype=torch.int64, device=dev) + rank * n
    eng.load_lists_device(1, glob.data_ptr(), row_ids.data_ptr(), X.data_ptr(), n)
    sizes = torch.bincount(assign.long(), minlength=nl).cpu().numpy()
    log(f"[rank {rank}] shard of {n} rows in {nl} lists (largest {sizes.max()}, median "
        f"{int(np.median(sizes))}) ready in {time.perf_counter() - t0:.1f}s")
    # queries from the union (the same on every rank): shard, then its mixture
    gq = torch.Generator(device=dev)
    gq.manual_seed(SEED + 500)
    nq_pool = 2 * B
    qshard = torch.randint(0, world, (nq_pool,), generator=gq, device=dev)
    Q = torch.empty((nq_pool, d), device=dev)
    for r in range(world):
        sel = torch.nonzero(qshard == r).flatten()
        if len(sel):
            Q[sel] = device_zipf_rows(means[r], len(sel), C4_ZIPF, SIGMA, SEED + 600 + r, dev)
    # exact global top-10 of 1024 queries: each rank's shard, merged over ranks
    qe = Q[:1024]
    best_s = best_i = None
    for b in range(0, n, 1 << 20):
        v, i = torch.topk(qe @ X[b:b + (1 << 20)].T, 10, dim=1)
        i = i + b
        if best_s is None:
            best_s, best_i = v, i
        else:
            cs, ci = torch.cat([best_s, v], 1), torch.cat([best_i, i], 1)
            best_s, o = torch.topk(cs, 10, dim=1)
            best_i = torch.gather(ci, 1, o)
    best_i = best_i + rank * n
    if world > 1:
        gs = torch.empty((world, 1024, 10), device=dev)
        gi = torch.empty((world, 1024, 10), dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(gs, best_s.contiguous())
        dist.all_gather_into_tensor(gi, best_i.contiguous())
        cs, ci = gs.permute(1, 0, 2).reshape(1024, -1), gi.permute(1, 0, 2).reshape(1024, -1)
        _, o = torch.topk(cs, 10, dim=1)
        exact = torch.gather(ci, 1, o).cpu().numpy()
    else:
        exact = best_i.cpu().numpy()
    del X, glob, row_ids, assign
    torch.cuda.empty_cache()
    sweep_p = (C4_NPROBE, 128, 256, 512)
    own = C4_BATCH_PER_GPU  # every rank brings its own batch per step
    sharded = ShardedSearch(eng, 1, K, own, world, dev, rank=rank, max_nprobe=max(sweep_p))

    def own_search(i, p):
        o = (i % 2) * B + rank * own
        return sharded.search_own_batch(Q[o:o + own], p)

    # recall@10 from nprobe 64 upward until it reaches 0.95 (skewed lists spread a
    # dense component's neighbours over many lists); rank 0's first batch holds the
    # queries with exact answers
    sweep = {}
    for p in sweep_p:
        ids, _, _ = own_search(0, p)
        torch.cuda.synchronize()
        r = recall_at_k(ids[:1024].cpu().numpy(), exact, K) if rank == 0 else 0.0
        if world > 1:
            t = torch.tensor([r], device=dev)
            dist.broadcast(t, 0)
            r = float(t.item())
        sweep[p] = r
        if sweep[p] >= 0.95:
            break
    nprobe = next((p for p in sweep if sweep[p] >= 0.95), max(sweep, key=sweep.get))
    recall = sweep[nprobe]
    eng.sync_errors()
    log(f"[rank {rank}] recall@10 by nprobe {sweep} -> nprobe {nprobe}")

    def step(i):
        own_search(i, nprobe)

    for w in range(args.warmup):
        step(w)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_selector(local_rank)) as clk:
        torch.cuda.nvtx.range_push("timed")
        ev0.record()
        for i in range(args.steps):
            step(i)
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    eng.sync_errors()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sharded.marks = []
    step(0)
    torch.cuda.synchronize()
    m = sharded.marks
    stage = {name: ea_eb for name, ea_eb in
             ((nm, ea.elapsed_time(eb)) for (_, ea), (nm, eb) in zip(m, m[1:]))}
    sharded.marks = None
    # one GPU: the engine's stage events and probed bytes over the same batches (the
    # blocking device call, outside the timed loop)
    eng_stage, roofline = {}, None
    if world == 1:
        ids_d = torch.empty((own, K), dtype=torch.int64, device=dev)
        sc_d = torch.empty((own, K), dtype=torch.float32, device=dev)
        cnt_d = torch.empty((own,), dtype=torch.int32, device=dev)
        eng.set_profiling(True)
        scan_ms, scan_bytes, streamed = [], [], []
        for i in range(4):
            o = (i % 2) * B
            eng.search_device(1, Q[o:o + own].data_ptr(), own, K, nprobe, ids_d.data_ptr(),
                              sc_d.data_ptr(), cnt_d.data_ptr())
            p = eng.last_profile()
            for key in ("ms_prep", "ms_coarse_gemm", "ms_select", "ms_worklist", "ms_scan",
                        "ms_merge", "ms_total"):
                eng_stage.setdefault(key[3:], []).append(p[key])
            scan_ms.append(p["ms_scan"])
            scan_bytes.append(p["scan_bytes"])
            streamed.append(p["streamed_bytes"])
        eng.set_profiling(False)
        eng_stage = {k: round(statistics.mean(v), 4) for k, v in eng_stage.items()}
        peak, peak_kind = peaks()
        achieved = statistics.mean(scan_bytes) / (statistics.mean(scan_ms) / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": None, "kernel": scan_kernel_name(),
                    "bytes_per_launch": statistics.mean(scan_bytes),
                    "streamed_bytes_per_launch": statistics.mean(streamed),
                    "streamed_gbs": statistics.mean(streamed) / (statistics.mean(scan_ms) / 1e3) / 1e9,
                    "ms_per_launch": statistics.mean(scan_ms),
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}
    if rank != 0:
        return
    qps = B * args.steps / (ms / 1e3)
    emit({
        "metric": "search QPS at recall@10>=0.95 (IVF, dim 1024, Zipf-skewed lists, "
                  "one 12.5M-row shard per GPU)",
        "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (per shard a seeded Zipf(1.1) mixture of 8192 components, on the GPU)",
        "config": {"workload": ("PROFILING CASE (not the 12.5M-row shard): " if args.c4_n else "")
                               + f"ivf-search: {world} x {n} x {d} fp32 unit-norm, cosine, "
                               f"nlist {world * nl}, nprobe {nprobe}, k {K}, batch {B}",
                   "rows_per_gpu": n, "nlist": world * nl, "nprobe": nprobe, "k": K,
                   "batch": B, "metric": "cosine (normalized)",
                   "scaling_protocol": "weak: one shard (rows, lists, 4096 queries) per GPU; "
                                       "N = 8 is the 100M-row, 65,536-list index",
                   "l2_flush": "not needed: each batch streams the shards (> 126 MB L2)"},
        "recall_at_10": recall, "recall_sweep": {str(p): r for p, r in sweep.items()},
        "stage_ms_rank0": {k: round(v, 4) for k, v in stage.items()},
        "stage_ms_engine": eng_stage or None,
        "parallelism": f"{world} shards; every GPU brings its own {own} queries per step: "
                       "batches all-gathered, probes selected per batch on its GPU and "
                       "all-gathered, per-shard top-k returned by one all-to-all"
                       if world > 1 else "1 GPU",
        "clocks": clk.summary(), "gpu_launches": None,
        "e2e": None, "roofline": roofline, "cpu_baseline": None,
    })


# ---------------------------------------------------------------- insert + split stream
# From the headline index: 1M new rows from shifted mixture means (offset
# N(0, 0.5^2) in norm), in batches of 8,192 routed by enqueue_insert_auto; after
# every batch one split pass (lists over 2x the mean size, 2-means, 5 rounds)
# and a 1,024-query search (k 10, nprobe 32).
C5_INSERT = 1_000_000
C5_BATCH = 8192
C5_SPLIT_FACTOR = 2.0
C5_SPLIT_ITERS = 5


def run_config5(args, rank, world, local_rank):
    import torch

    from m3_memory_b200 import cabi
    from m3_memory_b200 import synthetic as S

    if world > 1:
        raise SystemExit("the insert + split stream runs on one GPU (one engine)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n_ins = args.c5_n or C5_INSERT
    rng = np.random.default_rng(SEED)
    means = S.mixture_means(NCOMP, DIM, rng)
    X, _ = S.gaussian_mixture(N_VEC, means, SIGMA, rng)
    Q, _ = S.gaussian_mixture(BATCH * NBATCH, means, SIGMA, rng)
    shifted = S.shifted_means(means, 0.5, np.random.default_rng(SEED + 5))
    Xi, _ = S.gaussian_mixture(n_ins, shifted, SIGMA, np.random.default_rng(SEED + 6))
    Qs, _ = S.gaussian_mixture(BATCH * NBATCH, shifted, SIGMA, np.random.default_rng(SEED + 7))
    eng = cabi.Engine()
    if args.tile_rows is not None:
        eng.set_scan_tile_rows(args.tile_rows)
    build_headline_index(eng, X)
    eng.start(2, 0)
    # searches alternate between the original and the shifted distribution
    Qd = torch.from_numpy(np.concatenate([Q, Qs]).reshape(-1, BATCH, DIM)).to(dev)
    ids_d = torch.empty((BATCH, K), dtype=torch.int64, device=dev)
    sc_d = torch.empty((BATCH, K), dtype=torch.float32, device=dev)
    cnt_d = torch.empty((BATCH,), dtype=torch.int32, device=dev)

    def search(i):
        eng.search_device(1, Qd[i % Qd.shape[0]].data_ptr(), BATCH, K, NPROBE, ids_d.data_ptr(),
                          sc_d.data_ptr(), cnt_d.data_ptr(),
                          torch.cuda.current_stream(dev).cuda_stream)

    nb = -(-n_ins // C5_BATCH)
    warm = min(args.warmup, nb)
    t_ins = t_split = 0.0
    s_ms = []
    splits = 0
    t_all = None
    for b in range(nb):
        if b == warm:
            torch.cuda.synchronize()
            t_all = time.perf_counter()
            t_ins = t_split = 0.0
            s_ms = []
        lo, hi = b * C5_BATCH, min(n_ins, (b + 1) * C5_BATCH)
        t0 = time.perf_counter()
        assert eng.enqueue_insert_auto(1, np.arange(N_VEC + lo, N_VEC + hi, dtype=np.int64), Xi[lo:hi])
        eng.flush()
        t1 = time.perf_counter()
        splits += eng.split_oversized(1, C5_SPLIT_FACTOR, C5_SPLIT_ITERS, 1000 + b)
        t2 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        search(b)
        ev1.record()
        torch.cuda.synchronize()
        t_ins += t1 - t0
        t_split += t2 - t1
        s_ms.append(ev0.elapsed_time(ev1))
    wall = time.perf_counter() - t_all
    eng.sync_errors()
    timed_rows = n_ins - warm * C5_BATCH
    nlist = eng.info(1)[3]
    # recall of the final index against exact search over every row
    Xall = torch.from_numpy(np.concatenate([X, Xi])).to(dev)
    qe = Qd[1]
    exact = exact_topk_ip(Xall, qe, K).cpu().numpy()
    del Xall
    got, _, _ = eng.search(1, qe.cpu().numpy(), K, NPROBE)
    recall = recall_at_k(got, exact, K)
    eng.stop()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as O

        if O.have_ref():
            # the reference's own insert path (enqueue_insert_auto + flush) on the same
            # centroids, a bounded batch
            eng_centroids = eng.centroids(1)
            re = O.RefEngine()
            re.start(2, 0)
            re.create_ivf(1, DIM, METRIC_IP, False, eng_centroids)
            m = 1024
            t0 = time.perf_counter()
            re.enqueue_insert_auto(1, np.arange(m, dtype=np.int64), Xi[:m])
            re.flush()
            v = m / (time.perf_counter() - t0)
            re.stop()
            cpu = {"value": v, "unit": "rows/s", "cores": 1, "kind": "reference",
                   "sample": f"one {m}-row enqueue_insert_auto + flush into the reference "
                             f"AsyncEngine over the final {len(eng_centroids)} centroids "
                             "(its routing is one thread)"}
    emit({
        "metric": "online insert+split stream: inserted rows/s with a 1,024-query search "
                  "after every 8,192-row batch",
        "value": timed_rows / wall, "unit": "rows/s", "n_gpus": 1, "steps": nb - warm,
        "warmup": warm, "ms_per_step": 1e3 * wall / max(nb - warm, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded mixture; inserts from means shifted by N(0, 0.5^2) in norm)",
        "config": {"workload": f"insert+split stream: {N_VEC // 1_000_000}M x {DIM} IP index, "
                               f"nlist {NLIST} at start, {n_ins} inserts in batches of "
                               f"{C5_BATCH}, split lists over {C5_SPLIT_FACTOR}x the mean "
                               f"(2-means, {C5_SPLIT_ITERS} rounds), search k {K} nprobe "
                               f"{NPROBE} batch {BATCH} after each batch",
                   "parallelism": "1 GPU"},
        "stream": {"insert_s": t_ins, "split_s": t_split, "search_ms_mean": statistics.mean(s_ms),
                   "search_qps_mean": BATCH / (statistics.mean(s_ms) / 1e3),
                   "splits": splits, "nlist_final": nlist, "recall_at_10_final": recall},
        "cpu_baseline": cpu,
        "e2e": {"value": timed_rows / wall, "unit": "rows/s",
                "h2d_bytes_per_step": C5_BATCH * DIM * 4, "d2h_bytes_per_step": 0,
                "path": "host rows through m3g_enqueue_insert_auto + m3g_flush + "
                        "m3g_split_oversized; searches on device queries"},
    })


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--coarse", choices=["split", "sharded", "replicated"], default="split",
                    help="N > 1: coarse selection of each rank's slice of the queries over all "
                         "centroids, probes all-gathered (split); per rank over its own "
                         "centroids (sharded); or of every query on every rank (replicated)")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak",
                    help="N > 1: every GPU brings its own batch of queries per step, the lists "
                         "sharded over the GPUs (weak); or one batch per step split over the "
                         "GPUs (strong)")
    ap.add_argument("--nvec", type=int, default=None,
                    help="profiling only: fewer vectors (the headline line uses 1M)")
    ap.add_argument("--nlist", type=int, default=None, help="profiling only: fewer lists")
    ap.add_argument("--nprobe", type=int, default=None, help="profiling only: other nprobe")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=2,
                    help="2: the headline (1M x 1024 fp32, IP); 3: 10M x 768 bf16-stored lists, "
                         "L2, nlist 16384, k 100, nprobe x batch sweep; 5: online insert + split "
                         "stream from the headline index; 4: Zipf-skewed 12.5M-row shard per GPU, "
                         "cosine, nlist 8192 per shard, nprobe 64 (weak scaling)")
    ap.add_argument("--c5-n", type=int, default=None, help="config 5, profiling only: inserts")
    ap.add_argument("--c4-n", type=int, default=None, help="config 4, profiling only: rows per GPU")
    ap.add_argument("--storage", choices=["bf16", "fp32"], default="bf16",
                    help="config 3: list storage")
    ap.add_argument("--c3-n", type=int, default=None, help="config 3, profiling only: rows")
    ap.add_argument("--c3-k", type=int, default=None, help="config 3, profiling only: k")
    ap.add_argument("--c3-nlist", type=int, default=None, help="config 3, profiling only: nlist")
    ap.add_argument("--tile-rows", type=int, default=None,
                    help="row tiles of long lists in the scan: rows per tile (multiple of 128), "
                         "0 automatic (the default), -1 none")
    args = ap.parse_args()
    keep_stdout_for_result()
    global N_VEC, NLIST, NPROBE, FIXED_NPROBE, WORKLOAD
    if args.nvec or args.nlist or args.nprobe:
        N_VEC = args.nvec or N_VEC
        NLIST = args.nlist or NLIST
        NPROBE = args.nprobe or NPROBE
        FIXED_NPROBE = args.nprobe is not None
        WORKLOAD = (f"PROFILING CASE (not headline): {N_VEC} x {DIM}, nlist {NLIST}, "
                    f"nprobe {NPROBE}")
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch.distributed as dist

    if world > 1:
        import datetime

        import torch

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config == 3:
            run_config3(args, rank, world, local_rank)
        elif args.config == 4:
            run_config4(args, rank, world, local_rank)
        elif args.config == 5:
            run_config5(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
