"""Writes Faiss IndexIVFFlat files for the import tests, from Faiss's published
serialization layout (faiss/impl/index_write.cpp: the "IwFl" index with a flat
quantizer and "ilar" array inverted lists).  faiss itself is not installed
here, so these files are the only fixtures of that path and its parity stays
unpinned against real Faiss output."""
from __future__ import annotations

import struct

import numpy as np

FAISS_IP, FAISS_L2 = 0, 1


def _header(d, ntotal, metric):
    return struct.pack("<iqqqBi", d, ntotal, 1 << 20, 1 << 20, 1, metric)


def write_ivfflat(path, centroids, lists, metric=FAISS_L2, sparse=False, direct_map=0,
                  quantizer_tag=None):
    """centroids [nlist, d] fp32; lists: per list (ids int64 [n], vecs fp32 [n, d])."""
    C = np.ascontiguousarray(centroids, np.float32)
    nlist, d = C.shape
    ntotal = sum(len(i) for i, _ in lists)
    out = bytearray()
    out += b"IwFl" + _header(d, ntotal, metric) + struct.pack("<QQ", nlist, 1)
    tag = quantizer_tag or (b"IxF2" if metric == FAISS_L2 else b"IxFI")
    out += tag + _header(d, nlist, metric) + struct.pack("<Q", nlist * d) + C.tobytes()
    dm = np.zeros(0, np.int64) if direct_map == 0 else np.arange(ntotal, dtype=np.int64)
    out += struct.pack("<BQ", direct_map, len(dm)) + dm.tobytes()
    if direct_map == 2:
        out += struct.pack("<Q", 0)
    out += b"ilar" + struct.pack("<QQ", nlist, d * 4)
    sizes = [len(i) for i, _ in lists]
    if sparse:
        pairs = [v for l, s in enumerate(sizes) if s for v in (l, s)]
        out += b"sprs" + struct.pack("<Q", len(pairs)) + np.asarray(pairs, np.uint64).tobytes()
    else:
        out += b"full" + struct.pack("<Q", nlist) + np.asarray(sizes, np.uint64).tobytes()
    for ids, vecs in lists:
        if len(ids):
            out += np.ascontiguousarray(vecs, np.float32).tobytes()
            out += np.ascontiguousarray(ids, np.int64).tobytes()
    with open(path, "wb") as f:
        f.write(bytes(out))
    return len(out)
