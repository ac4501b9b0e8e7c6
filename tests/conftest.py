"""Test configuration: GPU tests are marked ``gpu`` and run only on a B200 box."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the sm_100a library")
    config.addinivalue_line("markers", "slow: CPU test that takes more than a few seconds")
    config.addinivalue_line("markers", "reference_gpu_arith: run the kernels in their default arithmetic "
                                       "(as the reference's compiled kernels), not the oracle's IEEE mode")


@pytest.fixture(autouse=True)
def _kernel_arithmetic(request):
    """GPU tests compare with the CPU oracle, which restates IEEE division and
    square root, so they run the kernels in that mode; tests marked
    ``reference_gpu_arith`` run the default mode. The default is restored after
    every GPU test."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    from lynnreal_omni_b200 import _lib
    _lib.set_arithmetic("reference_gpu" if request.node.get_closest_marker("reference_gpu_arith") else "ieee")
    yield
    _lib.set_arithmetic("reference_gpu")
