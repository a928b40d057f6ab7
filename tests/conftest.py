"""Test configuration.

* ``gpu`` marks tests that need a B200 and the built libcie_attn.so; they are
  the parity tests proper and call the CUDA path through the C ABI.
* Everything else runs on CPU: the oracle against the reference's golden
  vectors, the host-side logic, and the library's exported symbols.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "custom-inference-engine_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("test marked gpu but CUDA is not available")
    from kernels import _lib

    _lib.load()  # raises loudly if the extension is missing
    return torch.device("cuda")
