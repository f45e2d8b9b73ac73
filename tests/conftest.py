import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"


@pytest.fixture(scope="session")
def dev():
    """Device 0 through the C ABI (GPU tests only; no skip: a GPU run without
    the library or the device must fail loudly)."""
    import torch
    from xnpu_b200 import hal
    torch.cuda.init()
    d = hal.Device.open_default()
    yield d
    d.close()


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Print every parity figure the GPU tests recorded (tests/parity.py):
    the floored max relative error the asserts use, the unfloored one and
    the count of outputs above 1e-2 unfloored."""
    try:
        import parity
    except ImportError:
        return
    lines = parity.summary_lines()
    if lines:
        terminalreporter.section("parity")
        for line in lines:
            terminalreporter.write_line(line)
