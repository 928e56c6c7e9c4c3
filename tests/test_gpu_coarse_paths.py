"""Both coarse-GEMM paths give the same exact selection: the tensor-core bf16x3
GEMM (default) and the SIMT fp32 GEMM (M3G_COARSE_GEMM=simt, checked in a child
process because the choice is read once per process)."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from gpu_common import engine_from_golden
from helpers import load_golden

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

CHILD = r'''
import sys, numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
from m3_memory_b200 import cabi
from gpu_common import engine_from_golden
from helpers import load_golden
out = {}
for case in ("ip_mixture", "l2_raw", "cosine_norm"):
    g = load_golden(case)
    e = engine_from_golden(cabi, g)
    out[case] = e.select_probes(1, g["Q"], 5)
    out[case + "_assign"] = e.nearest_clusters(1, g["lvecs"])
np.savez(sys.argv[2], **out)
'''


def test_simt_and_tensor_core_paths_agree(cuda_ok, tmp_path):
    from m3_memory_b200 import cabi

    f = tmp_path / "simt.npz"
    env = dict(os.environ, M3G_COARSE_GEMM="simt")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), str(f)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    simt = np.load(f)
    for case in ("ip_mixture", "l2_raw", "cosine_norm"):
        g = load_golden(case)
        e = engine_from_golden(cabi, g)
        np.testing.assert_array_equal(e.select_probes(1, g["Q"], 5), simt[case])
        np.testing.assert_array_equal(e.nearest_clusters(1, g["lvecs"]), simt[case + "_assign"])
