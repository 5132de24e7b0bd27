"""Shared pytest configuration.

Markers:
  gpu  — needs a CUDA device (sm_100a); run with ``-m gpu`` on a B200.
Everything unmarked runs on a CPU-only host.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


def _ensure_extension():
    try:
        import squish_b200._C  # noqa: F401
        return
    except ImportError:
        pass
    subprocess.run([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=ROOT, check=True,
                   stdout=subprocess.DEVNULL)


_ensure_extension()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
