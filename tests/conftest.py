"""Shared pytest configuration.

`-m gpu` tests need a B200 and the built libraries; everything else runs on
CPU. The repository root is put on sys.path so `zcutlass_b200`, `oracle` and
the drop-in `zcutlass_torch` / `zcutlass_vllm` packages import without
installation.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"tests target sm_100a (B200); found sm_{major}{minor}"
    return torch.device("cuda", 0)
