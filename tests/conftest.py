"""Test configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs the CPU suite (oracle against golden fixtures, host logic,
C-ABI exports). `-m gpu` runs the parity tests through the C ABI on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = ROOT / "qwen3-tts-rsi-engine_b200"
for path in (ROOT, PACKAGE_ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from qwen3_tts_b200 import _lib
    _lib.load()  # fail loudly if the kernels are not built
    return torch.device("cuda:0")
