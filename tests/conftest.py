import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


@pytest.fixture(scope="session")
def b200_ops():
    """GPU fixture: FAILS (never skips) when a GPU is present but the native
    library does not load, so a GPU run cannot pass on a fallback."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from vllm_sm70_b200 import _ext

    assert _ext.load(), f"_b200_C failed to load on a GPU machine: {_ext.error()}"
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    torch.ops._b200_C.init_device(torch.cuda.current_device())
    from vllm_sm70_b200.ops import linear

    linear.configure_workspace(torch.cuda.current_device())
    return torch.ops._b200_C


@pytest.fixture(autouse=True)
def _check_device_status(request):
    """After every GPU test, the bounded-wait status word must be clean."""
    yield
    if request.node.get_closest_marker("gpu") and torch.cuda.is_available():
        from vllm_sm70_b200 import _ext

        if _ext.loaded():
            torch.cuda.synchronize()
            st = int(torch.ops._b200_C.read_status(torch.cuda.current_device(), True))
            assert st == 0, f"kernel status word set: {st}"


def max_abs_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-6))


@pytest.fixture
def rel_err():
    return max_abs_rel
