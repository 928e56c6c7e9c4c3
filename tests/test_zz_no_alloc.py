"""The selection entry point for callers that cannot allocate GPU memory.

m3g_select_probes_noalloc keeps its scratch in a fixed array inside the library
instead of allocating, for processes that own all device memory up front or
must not let the library synchronise the device through cudaMalloc / cudaFree.
Its answer must equal the engine's m3g_select_probes on the same inputs, call
after call (the shared scratch keeps the previous call's contents).

This file is collected last on purpose: a failure here should not hide the
results of the other GPU tests in a run that stops at the first failure.
"""
import numpy as np
import pytest

from helpers import load_golden

pytestmark = pytest.mark.gpu


def _engine_probes(cabi, g, nprobe):
    e = cabi.Engine()
    C = g["C"]
    e.create_ivf(1, C.shape[1], int(g["metric"]), bool(g["normalized"]), C)
    return e.select_probes(1, g["Q"], nprobe)


def _noalloc_probes(cabi, torch, g, nprobe):
    Q = torch.from_numpy(np.ascontiguousarray(g["Q"], np.float32)).cuda()
    C = torch.from_numpy(np.ascontiguousarray(g["C"], np.float32)).cuda()
    P = min(nprobe, C.shape[0]) if nprobe > 0 else C.shape[0]
    out = torch.full((Q.shape[0], P), -7, dtype=torch.int32, device="cuda")
    cabi.select_probes_noalloc(Q.data_ptr(), Q.shape[0], C.data_ptr(), C.shape[0], C.shape[1],
                               int(g["metric"]), bool(g["normalized"]), nprobe, out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _same_selection(oracle_mod, g, got, want):
    """Equal, or different only where the exact scores tie."""
    O = oracle_mod
    metric, norm = int(g["metric"]), bool(g["normalized"])
    for q in range(len(g["Q"])):
        if not np.array_equal(got[q], want[q]):
            s_got = [O.score(g["Q"][q], g["C"][c], metric, norm) for c in got[q]]
            s_want = [O.score(g["Q"][q], g["C"][c], metric, norm) for c in want[q]]
            assert s_got == s_want, (q, got[q], want[q])


def test_noalloc_matches_engine_on_consecutive_calls(cuda_ok, oracle_mod):
    import torch

    from m3_memory_b200 import cabi

    cases = [("ip_mixture", 3), ("l2_raw", 5), ("cosine_raw_zero", 2), ("ip_mixture", 8)]
    for name, nprobe in cases:  # back to back: each call reuses the shared scratch
        g = load_golden(name)
        got = _noalloc_probes(cabi, torch, g, nprobe)
        want = _engine_probes(cabi, g, nprobe)
        assert got.shape == want.shape
        _same_selection(oracle_mod, g, got, want)


def _synthetic(nq, L, d, metric, normalized, seed):
    rng = np.random.default_rng(seed)
    means = rng.standard_normal((12, d)).astype(np.float32)
    C = (means[rng.integers(0, 12, L)] + 0.3 * rng.standard_normal((L, d))).astype(np.float32)
    Q = (means[rng.integers(0, 12, nq)] + 0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    if normalized:
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return {"Q": Q, "C": C, "metric": metric, "normalized": normalized}


def test_noalloc_more_shapes(cuda_ok, oracle_mod):
    """The large-P selection kernel (P = 200 and P = 1500 > 1024, returned in id
    order), a call within 1 KB of the fixed scratch's end, a call enqueued on a
    caller's stream, and the normalised-cosine golden case."""
    import torch

    from m3_memory_b200 import cabi

    cases = [(_synthetic(24, 2048, 64, 1, False, 1), 200),
             (_synthetic(12, 2048, 32, 0, False, 2), 1500),
             (_synthetic(1024, 4085, 16, 1, False, 3), 8),  # needs 4193280 of 4194304 floats
             (load_golden("cosine_norm"), 6)]
    for g, nprobe in cases:
        got = _noalloc_probes(cabi, torch, g, nprobe)
        want = _engine_probes(cabi, g, nprobe)
        assert got.shape == want.shape
        if nprobe > 1024:  # above 1024 the set comes back in id order
            for q in range(len(got)):
                np.testing.assert_array_equal(np.sort(got[q]), np.sort(want[q]))
        else:
            _same_selection(oracle_mod, g, got, want)
    # enqueued on a caller's non-blocking stream
    g = cases[0][0]
    Q = torch.from_numpy(g["Q"]).cuda()
    C = torch.from_numpy(g["C"]).cuda()
    out = torch.full((len(g["Q"]), 32), -7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    cabi.select_probes_noalloc(Q.data_ptr(), Q.shape[0], C.data_ptr(), C.shape[0], C.shape[1],
                               1, False, 32, out.data_ptr(), s.cuda_stream)
    s.synchronize()
    _same_selection(oracle_mod, g, out.cpu().numpy(), _engine_probes(cabi, g, 32))


def test_noalloc_limits(cuda_ok):
    import torch

    from m3_memory_b200 import cabi

    Q = torch.zeros((4096, 8), dtype=torch.float32, device="cuda")
    C = torch.zeros((2048, 8), dtype=torch.float32, device="cuda")
    out = torch.empty((4096, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(cabi.M3GError) as ei:  # 4096 x 2048 scores exceed the fixed scratch
        cabi.select_probes_noalloc(Q.data_ptr(), 4096, C.data_ptr(), 2048, 8, cabi.IP, False, 4,
                                   out.data_ptr())
    assert ei.value.code == cabi.M3G_EUNSUPPORTED
    with pytest.raises(ValueError):  # dim must be a multiple of 4
        cabi.select_probes_noalloc(Q.data_ptr(), 16, C.data_ptr(), 16, 6, cabi.IP, False, 4,
                                   out.data_ptr())
