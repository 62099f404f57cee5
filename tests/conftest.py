import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def dev():
    import torch
    if not cuda_ok():
        pytest.skip("no sm_100 GPU")
    from catfuse_b200 import _lib
    _lib.load()
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_error_word(request):
    """GPU tests run with the networks' per-forward error check on, and after
    each one the bounded-wait error word must be clear (an expired wait would
    otherwise leave wrong tensors without an exception)."""
    if request.node.get_closest_marker("gpu") is None or not cuda_ok():
        yield
        return
    from catfuse_b200 import ops
    from catfuse_b200.network import CTFNetwork
    from catfuse_b200.spikformer_net import CTFSpikformer
    CTFNetwork.check_errors = True
    CTFSpikformer.check_errors = True
    yield
    ops.check_device_error()
