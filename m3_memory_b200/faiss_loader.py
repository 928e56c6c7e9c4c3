"""``rebuild_from_faiss`` with the reference's signature
(AgentMemory/M3/faiss_loader.py:24-79): rebuild an engine index from a Faiss
IVF dump.

The reference reads the file with the ``faiss`` package and calls
``create_ivf`` + ``load_cluster`` per list.  Here the engine reads the file
itself (``m3g_rebuild_from_faiss``, a parser of Faiss's published
IndexIVFFlat layout), so neither faiss nor a host-side copy of the vectors
through Python is needed; the lists go straight into the device arenas.
Supported input: a plain IndexIVFFlat (float codes) with a flat quantizer,
metric L2 or inner product -- the same cases the reference's loader accepts
short of IVF indexes nested inside other Faiss wrappers.
"""
from __future__ import annotations

from pathlib import Path

__all__ = ["rebuild_from_faiss"]


def rebuild_from_faiss(engine, *, index_id: int, path, normalized: bool = True,
                       storage: str = "fp32") -> None:
    """Replace ``index_id`` of ``engine`` (the ``_m3_async.AsyncEngine`` or a
    ``cabi.Engine``) with the index stored in the Faiss file ``path``."""
    path = Path(path)
    if not path.is_file():
        raise FileNotFoundError(f"Faiss index file not found: {path}")
    if hasattr(engine, "h"):  # ctypes binding
        from . import cabi

        engine.rebuild_from_faiss(int(index_id), str(path), bool(normalized),
                                  cabi.BF16 if storage == "bf16" else cabi.F32)
    else:
        engine.rebuild_from_faiss(int(index_id), str(path), bool(normalized), storage)
