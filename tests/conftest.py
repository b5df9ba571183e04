"""Test configuration.

Markers:
  gpu   -- needs a CUDA device (a B200); the CPU tier runs `-m "not gpu"`.
  slow  -- multi-process or long-running CPU tests.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: multi-process or long-running CPU test")


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def pytest_sessionstart(session):
    # Opt-in native backtrace of a host crash (diagnostics only).
    if os.environ.get("EWB_SEGV_BT") == "1":
        try:
            from elysium_wan_b200.ops import _ext

            _ext.ext().install_segv_backtrace()
        except Exception:
            pass
