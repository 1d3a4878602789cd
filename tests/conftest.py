import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; parity tests through the C ABI")
    config.addinivalue_line("markers", "slow: long-running (full-size) cases")


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import Port
    return Port()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Ref
    try:
        return Ref()
    except (FileNotFoundError, OSError) as e:
        pytest.skip(f"reference host backend not available: {e}")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    from alpaka3_b200 import capi
    capi.lib()  # the CUDA path must load; no fallback
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
