"""Test configuration: GPU tests are marked ``gpu`` and run only on a B200 box."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the sm_100a library")
    config.addinivalue_line("markers", "slow: CPU test that takes more than a few seconds")
