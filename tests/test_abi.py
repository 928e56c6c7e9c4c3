"""The drop-in boundary on a CPU-only box: libm3gpu loads and exports every
symbol include/m3gpu.h declares; the pybind module `_m3_async` carries the
reference's class, enum and method names; host-side argument checks fire
before any device work."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "m3gpu.h").read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(m3g_[a-z_]+)\s*\(", text, re.M)))


def test_header_symbols_exported():
    from m3_memory_b200 import cabi

    lib = cabi.lib()
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes table covers them all
    assert set(names) == set(cabi.SIGNATURES), set(names) ^ set(cabi.SIGNATURES)


def test_version_and_null_handle():
    from m3_memory_b200 import cabi

    assert cabi.lib().m3g_version() >= 100
    rc = cabi.lib().m3g_flush(None)
    assert rc == cabi.M3G_EINVAL
    assert b"null" in cabi.lib().m3g_last_error()


def test_pybind_surface_matches_reference():
    from m3_memory_b200 import load

    m = load()
    # Metric enum values, bindings_async.cpp:17-21
    assert int(m.Metric.L2) == 0 and int(m.Metric.IP) == 1 and int(m.Metric.COSINE) == 2
    assert m.L2 == m.Metric.L2  # export_values()
    ref_methods = ["start", "stop", "create_ivf", "set_queue_policy", "set_search_policy",
                   "set_maintenance_policy", "enqueue_insert", "enqueue_insert_auto",
                   "enqueue_update", "enqueue_delete", "load_cluster", "flush", "search",
                   "dim_of", "metric_of", "normalized_of", "nlist_of"]
    for name in ref_methods:
        assert hasattr(m.AsyncEngine, name), name
    doc = m.AsyncEngine.search.__doc__
    assert "nprobe" in doc and "k" in doc  # both overloads


def test_info_defaults_for_unknown_index():
    """m3_async.cpp:317-351: unknown index -> dim 0, COSINE, normalized, 0 lists."""
    from m3_memory_b200 import load

    m = load()
    e = m.AsyncEngine()
    assert e.dim_of(5) == 0
    assert e.metric_of(5) == m.Metric.COSINE
    assert e.normalized_of(5) is True
    assert e.nlist_of(5) == 0


def test_binding_shape_checks_before_device_work():
    """The reference binding's shape errors (bindings_async.cpp), raised as RuntimeError."""
    from m3_memory_b200 import load

    m = load()
    e = m.AsyncEngine()
    with pytest.raises(RuntimeError, match="queries must be 2D"):
        e.search(0, np.zeros(4, np.float32), 3)
    with pytest.raises(RuntimeError, match="unknown index_id"):
        e.search(0, np.zeros((1, 4), np.float32), 3)
    with pytest.raises(RuntimeError, match="centroids must be 2D"):
        e.create_ivf(0, 4, m.Metric.L2, False, np.zeros(4, np.float32))
    with pytest.raises(RuntimeError, match="centroids dim mismatch"):
        e.create_ivf(0, 4, m.Metric.L2, False, np.zeros((2, 3), np.float32))
    with pytest.raises(RuntimeError, match="ids must be 1D"):
        e.enqueue_insert(0, 0, np.zeros((2, 2), np.int64), np.zeros((2, 4), np.float32))
    with pytest.raises(RuntimeError, match="ids.size != vectors.N"):
        e.enqueue_insert_auto(0, np.zeros(3, np.int64), np.zeros((2, 4), np.float32))
    with pytest.raises(RuntimeError, match="unknown index_id"):
        e.load_cluster(0, 0, np.zeros(2, np.int64), np.zeros((2, 4), np.float32))


def test_queue_semantics_without_start():
    """enqueue_* returns False while the engine is stopped (m3_async.cpp:132-135)."""
    from m3_memory_b200 import cabi

    e = cabi.Engine()
    # deletes need no index (the reference binding does not check, :248-271)
    assert e.enqueue_delete(3, 0, np.arange(4)) is False
    e.flush()  # returns at once when not running (m3_async.cpp:193)
