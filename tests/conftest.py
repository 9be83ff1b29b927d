"""Test configuration: the ``gpu`` marker and shared paths.

``-m "not gpu"`` runs the oracle-vs-golden pins, host logic and library-load checks on the CPU;
``-m gpu`` runs the CUDA parity tests (they need a B200 and the built extension).
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def reference_project():
    """The reference project directory (the one holding the ``heimdall`` package), from the environment
    variable HEIMDALL_REFERENCE; None when it is unset or does not exist (tests that need it skip)."""
    p = os.environ.get("HEIMDALL_REFERENCE")
    if not p:
        return None
    path = Path(p)
    if (path / "Heimdall" / "heimdall").is_dir():
        path = path / "Heimdall"
    return path if (path / "heimdall").is_dir() else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built extension")


@pytest.fixture(scope="session")
def golden_retrieval():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "golden_retrieval.pt", weights_only=False)


@pytest.fixture(scope="session")
def golden_gdn():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "golden_gdn.pt", weights_only=False)


@pytest.fixture(scope="session")
def golden_forward():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "golden_forward.pt", weights_only=False)


@pytest.fixture(scope="session")
def golden_layer():
    import torch
    return torch.load(ROOT / "tests" / "golden" / "golden_layer.pt", weights_only=False)


@pytest.fixture(autouse=True)
def _no_device_timeouts(request):
    """GPU tests must leave the device error record clean (no bounded wait gave up)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from heimdall_b200 import _lib
    rec = _lib.device_error(torch.cuda.current_stream().cuda_stream)
    assert rec[0] == 0, f"a device-side wait gave up: site 0x{rec[0] >> 8:x}, block ({rec[1]}, {rec[2]}), thread {rec[3]}"
