"""pytest setup: marker registration and import paths.

`-m "not gpu"` runs the oracle KATs, host-logic and C-ABI load/export checks
on CPU; `-m gpu` runs the parity tests through the C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "forge-gpu_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden"),
          ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and libforge_sph.so")


@pytest.fixture(scope="session")
def cuda():
    """Torch with a CUDA device; GPU tests fail loudly (no silent skip) if absent."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import forge_sph
    forge_sph.lib()
    return torch
