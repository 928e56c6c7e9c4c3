"""m3_memory_b200 -- B200-native (sm_100a) engine for the M3 IVF index hot path of
AgentMemory's `m3` backend.

* ``m3_memory_b200._m3_async`` is the drop-in replacement of the reference's
  pybind module ``AgentMemory.M3._m3_async`` (``Metric``, ``AsyncEngine``).
* ``m3_memory_b200.cabi`` binds the C ABI of ``libm3gpu.so`` (include/m3gpu.h).
* ``m3_memory_b200.synthetic`` holds the seeded workload generators.

The compiled pieces are built in-tree by ``python -m m3_memory_b200._build``.
Importing ``_m3_async`` without them raises: there is no CPU fallback.
"""
from pathlib import Path

__all__ = ["PKG_DIR", "load"]

PKG_DIR = Path(__file__).resolve().parent


def load():
    """Returns the compiled ``_m3_async`` module (raises ImportError if unbuilt)."""
    from . import _m3_async  # noqa: F401  (compiled extension)

    return _m3_async
