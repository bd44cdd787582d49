"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs the oracle-vs-golden checks, host logic and the
library-loading checks on CPU; `-m gpu` runs the CUDA parity tests, which
call the kernels through the C ABI of libgrs_b200.so.
"""
from __future__ import annotations

from pathlib import Path
import sys

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libgrs_b200.so")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
