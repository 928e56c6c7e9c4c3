"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on a CPU-only box: the oracle against the golden fixtures
and the reference core, the C-ABI surface, and host-side logic.  `-m gpu`
runs the parity tests proper, which call the CUDA engine through its C ABI.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O

    if not O.C_LIB.is_file():
        O.build(ref=None)
    return O


@pytest.fixture(scope="session")
def have_ref(oracle_mod):
    if not oracle_mod.have_ref():
        try:
            oracle_mod.build(ref=None)
        except Exception:
            pass
    return oracle_mod.have_ref()


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    return True
