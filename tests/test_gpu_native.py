"""Runs the native C++ API test (tests/native/test_gemm_api.cpp): the C++
entry points (zcutlass::gemm with GemmDesc and with GemmArguments, validation
codes, zero sizes, selection telemetry) against the CPU oracle."""

from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

NATIVE = Path(__file__).resolve().parent / "native"


def _build() -> Path:
    subprocess.run(["make", "-s", "-C", str(NATIVE)], check=True)
    return NATIVE / "zcutlass_api_test"


def test_native_test_builds():
    assert _build().exists()


@pytest.mark.gpu
def test_native_cpp_api(cuda_device):
    r = subprocess.run([str(_build())], capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:])
    assert r.returncode == 0, r.stdout[-6000:] + r.stderr[-2000:]
    assert "0 failures" in r.stdout
