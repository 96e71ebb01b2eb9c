"""Test configuration: the ``gpu`` marker, and import paths for the package and the oracle."""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "qwen-image21-tensorfold-rtx_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libtfb.so")


import pytest  # noqa: E402


@pytest.fixture
def dev():
    """cuda:0 for GPU tests; after the test the kernels' device error word must be clean (no wait ran out)."""
    import torch

    from tfimage import _lib

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    yield torch.device("cuda:0")
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True) == 0, "a kernel pipeline wait ran out"
