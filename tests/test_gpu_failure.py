"""Failure detection on the GPU without a fault.

A kernel whose bounded mbarrier wait is never satisfied (nothing arrives)
must give up after its limit, record an error code that the host reads, and
return; the device must stay usable for the next GEMM.
"""

from __future__ import annotations

import time

import pytest

from gemm_case import Case, check_case
from oracle import oracle
from zcutlass_b200 import _native


@pytest.mark.gpu
def test_bounded_wait_expires_and_reports(cuda_device):
    assert _native.device_error(clear=True) == 0
    t0 = time.perf_counter()
    code = _native.lib().zcutlass_selftest_bounded_wait(20000)  # 20 ms limit
    elapsed = time.perf_counter() - t0
    assert code == (15 << 4) | 15, code
    assert elapsed < 5.0
    assert _native.device_error(clear=True) == 0  # the self test cleared it
    # the context is still healthy: a normal GEMM runs and checks out
    check_case(Case("after timeout", oracle.BF16, 300, 520, 264, 1.0, 0.0, True, gen="normal"))
