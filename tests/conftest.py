import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built sm_100a library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def pytest_sessionfinish(session, exitstatus):
    """With HC_PARITY_REPORT set, write the selection comparisons of the
    session (flips, boundary ties, set differences per test) as JSON there."""
    path = os.environ.get("HC_PARITY_REPORT")
    if not path:
        return
    try:
        import parity
    except Exception:
        return
    if not parity.RECORDS:
        return
    import json
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump({"summary": parity.summary(), "records": parity.RECORDS}, f, indent=1)
