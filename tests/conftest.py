"""Test configuration.

Two kinds of tests:
- unmarked tests run on the CPU: the oracle against the reference's golden
  vectors and known answers, host-side logic, the C ABI library's exports, and
  multi-process ES logic on gloo ranks;
- `@pytest.mark.gpu` tests call the CUDA library through its C ABI (via the
  drop-in modules) on a B200 and compare every output with the oracle.

The drop-in modules live in the flat directory metal-rl-envs_b200/ (imported by
bare name, as the reference's modules are); the oracle is the package `oracle`
at the repository root.
"""

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "metal-rl-envs_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"

for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels through the C ABI")


def golden(name):
    """The arrays of tests/golden/<name>.npz as a dict."""
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests; fails (does not skip) when there is none, since a GPU
    test that silently skips would hide a missing native path."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    import rlenv_lib

    rlenv_lib.load()
    return torch.device("cuda", 0)
