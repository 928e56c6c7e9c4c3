"""The device-side failure path, exercised without faulting or hanging the GPU:
m3g_set_test_wait_limit makes one bounded mbarrier wait of the tensor-core
scan run out (its barrier is never completed), so the search must come back
with M3G_ETIMEOUT, and the engine must answer correctly again once the hook is
off (every role left, nothing was left in flight, TMEM was freed)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_expired_device_wait_reports_timeout_and_recovers(cuda_ok):
    import torch

    from m3_memory_b200 import cabi

    rng = np.random.default_rng(9)
    L, d = 16, 64
    C = rng.standard_normal((L, d)).astype(np.float32)
    a = rng.integers(0, L, 4000)
    X = (C[a] + 0.3 * rng.standard_normal((4000, d))).astype(np.float32)
    e = cabi.Engine()
    e.create_ivf(1, d, cabi.IP, False, C)
    for c in range(L):
        rows = np.flatnonzero(a == c)
        e.load_cluster(1, c, rows.astype(np.int64), X[rows])
    Q = (C[rng.integers(0, L, 50)] + 0.3 * rng.standard_normal((50, d))).astype(np.float32)
    want = e.search(1, Q, 10, 4)
    for ns in (1_000, 200_000):
        e.set_test_wait_limit(ns)
        with pytest.raises(cabi.M3GError) as ei:
            e.search(1, Q, 10, 4)
        assert ei.value.code == cabi.M3G_ETIMEOUT
        # also through the device path, reported by m3g_sync_errors
        qd = torch.from_numpy(Q).cuda()
        ids = torch.empty((50, 10), dtype=torch.int64, device="cuda")
        sc = torch.empty((50, 10), dtype=torch.float32, device="cuda")
        cnt = torch.empty((50,), dtype=torch.int32, device="cuda")
        s = torch.cuda.Stream()
        with pytest.raises(cabi.M3GError) as ei:
            e.search_device(1, qd.data_ptr(), 50, 10, 4, ids.data_ptr(), sc.data_ptr(),
                            cnt.data_ptr(), s.cuda_stream)
            s.synchronize()
            e.sync_errors()
        assert ei.value.code == cabi.M3G_ETIMEOUT
    e.set_test_wait_limit(0)
    got = e.search(1, Q, 10, 4)
    for x, y in zip(got, want):
        np.testing.assert_array_equal(x, y)
