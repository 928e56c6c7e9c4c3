"""Helpers for the GPU parity tests: build engine indexes from golden cases."""
import numpy as np

from helpers import lists_of


def engine_from_golden(cabi, g, index_id=1, engine=None, start=True):
    e = engine or cabi.Engine()
    C = g["C"]
    d = C.shape[1]
    e.create_ivf(index_id, d, int(g["metric"]), bool(g["normalized"]), C)
    off, vecs, ids, alive = lists_of(g)
    for c in range(len(off) - 1):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            e.load_cluster(index_id, c, ids[b:t], vecs[b:t])
    if (alive == 0).any():
        if start:
            e.start(1, 0)
        for c in range(len(off) - 1):
            b, t = int(off[c]), int(off[c + 1])
            dead = ids[b:t][alive[b:t] == 0]
            if len(dead):
                assert e.enqueue_delete(index_id, c, dead)
        e.flush()
    return e


def expected_probes(O, Q, C, metric, normalized, p):
    return np.stack([O.select_nprobe(q, C, metric, normalized, p) for q in Q])
