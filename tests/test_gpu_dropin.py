"""The drop-in module `_m3_async` used the way M3Backend uses the reference's
(AgentMemory/backend/m3.py): create_ivf, enqueue_insert_auto, flush, search."""
import numpy as np
import pytest

from helpers import load_golden

pytestmark = pytest.mark.gpu


def test_backend_style_flow(cuda_ok, oracle_mod, have_ref):
    from m3_memory_b200 import load

    m = load()
    g = load_golden("cosine_norm")
    eng = m.AsyncEngine()
    eng.start(2, 1)
    d = g["C"].shape[1]
    eng.create_ivf(7, d, m.Metric.COSINE, True, g["C"])
    assert eng.dim_of(7) == d and eng.nlist_of(7) == len(g["C"])
    assert eng.metric_of(7) == m.Metric.COSINE and eng.normalized_of(7)
    assert eng.enqueue_insert_auto(7, g["lids"], g["lvecs"])
    eng.flush()
    out_ids, out_scores = eng.search(7, g["Q"], 10, 32)
    assert isinstance(out_ids, list) and isinstance(out_ids[0], list)
    assert len(out_ids) == len(g["Q"]) and all(len(r) == 10 for r in out_ids)
    ref_ids = g["ref_ids_p32"]
    hits = sum(len(set(a) & set(b.tolist())) for a, b in zip(out_ids, ref_ids))
    assert hits / ref_ids.size >= 0.999
    # search(index, q, k) uses the default nprobe (8)
    a_ids, _ = eng.search(7, g["Q"][:5], 3)
    b_ids, _ = eng.search(7, g["Q"][:5], 3, 8)
    assert a_ids == b_ids
    with pytest.raises(RuntimeError, match="query dim mismatch"):
        eng.search(7, np.zeros((1, d + 1), np.float32), 3)
    eng.stop()


def test_device_fast_path_matches_host(cuda_ok):
    import torch

    from m3_memory_b200 import load

    m = load()
    g = load_golden("ip_mixture")
    eng = m.AsyncEngine()
    d = g["C"].shape[1]
    eng.create_ivf(1, d, m.Metric.IP, False, g["C"])
    off = g["off"]
    for c in range(len(off) - 1):
        b, t = int(off[c]), int(off[c + 1])
        if t > b:
            eng.load_cluster(1, c, g["lids"][b:t], g["lvecs"][b:t])
    Q = torch.from_numpy(g["Q"]).cuda()
    nq, k = Q.shape[0], 10
    ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    sc = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    cnt = torch.empty((nq,), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    eng.search_into_device(1, Q.data_ptr(), nq, k, 3, ids.data_ptr(), sc.data_ptr(),
                           cnt.data_ptr(), stream)
    eng.sync_errors()
    torch.cuda.synchronize()
    h_ids, h_sc = eng.search(1, g["Q"], k, 3)
    assert ids.cpu().numpy().tolist() == h_ids
    np.testing.assert_array_equal(sc.cpu().numpy(), np.array(h_sc, np.float32))
